"""Benchmark evaluation: dataset registry, runner, CLI (reference ``src/synthefy_nori/evaluation``)."""
