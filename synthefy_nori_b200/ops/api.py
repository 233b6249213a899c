def _placeholder(): pass
