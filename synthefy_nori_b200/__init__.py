"""Nori on Blackwell: a B200-native tabular foundation model framework."""

__version__ = "0.1.0"
