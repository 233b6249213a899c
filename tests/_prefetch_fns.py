"""Picklable batch generators for the prefetcher tests (importable by spawned workers)."""

import os

import numpy as np


def make_batch(seed):
    return np.random.default_rng(seed).standard_normal(4)


def failing(seed):
    if seed == 2:
        raise ValueError("bad table")
    return seed


def dying(seed):
    os._exit(3)  # the process ends without reporting
