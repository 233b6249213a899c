"""Memory policy for the context cache (reference ``inference/memory_policy.py``).

The context K/V cache - not the model - is what exhausts GPU memory on large tables
(``L * (G+1) * N * 2 * E`` elements, reference ``memory_policy.py:368-389``).
``MemoryPolicy`` is the user-facing contract: the same field names, presets
(``"exact"``, ``"max_context"``, ``"off"``) and coercion rules (``None`` / preset name /
dict / instance) as the reference, so configurations carry over. ``resolve`` picks the
rung for a given table and device:

    no_cache -> resident_bf16 -> resident_int8 -> context_sharded_int8 -> subsample

``context_sharded_int8`` is this build's multi-GPU rung (the cache split by context rows
over the GPUs of one node, ``parallel/context_parallel.py``). The reference's host-offload
and streamed rungs (``offload_*``, ``stream_*``) are accepted in configurations but not
provided here: with 180 GB per B200 and the sharded rung they are not needed on this
hardware, and asking for them explicitly raises.
"""

from __future__ import annotations

from typing import Literal

from pydantic import BaseModel, ConfigDict, Field, field_validator

CacheDtype = Literal["bf16", "int8"]
MEMORY_PRESETS = ("exact", "max_context", "off")
RUNGS = ("no_cache", "resident_bf16", "resident_int8", "context_sharded_int8", "subsample", "plain_loop")
KV_TENSORS_PER_ROW = 2
BYTES_PER_GIB = 1024 ** 3


def estimate_cache_gb(*, n_context_rows: int, n_groups: int, nlayers: int, embed_dim: int,
                      bytes_per_element: int = 2) -> float:
    """Context cache footprint in GiB (``n_groups`` counts the target token too)."""
    return nlayers * n_groups * n_context_rows * KV_TENSORS_PER_ROW * embed_dim * bytes_per_element / BYTES_PER_GIB


def int8_footprint_gb(est_bf16_gb: float, *, head_dim: int) -> float:
    """The same cache stored int8 with one fp32 scale per (token, head) vector."""
    return est_bf16_gb / 2.0 * (1.0 + 4.0 / max(head_dim, 1))


class MemoryPolicy(BaseModel):
    """How ``predict`` may spend GPU memory on the context cache."""

    model_config = ConfigDict(extra="forbid", frozen=True)

    cache: bool = Field(True, description="build a context K/V cache (False: recompute the context per query chunk)")
    reuse_context_cache: bool = Field(True, description="keep the cache across predict calls with the same context")
    cache_dtype: CacheDtype = Field("bf16", description="starting precision of the cache")
    allow_quantization: bool = Field(True, description="may fall back from bf16 to int8 when bf16 does not fit")
    gpu_budget_frac: float = Field(0.6, gt=0.0, le=1.0, description="fraction of device memory the cache may use")
    gpu_budget_absolute_gb: float | None = Field(None, gt=0.0)
    offload_to_host: bool = Field(False, description="reference host-offload rung (not provided by this build)")
    host_budget_frac: float = Field(0.5, gt=0.0, le=1.0)
    host_budget_absolute_gb: float | None = Field(None, gt=0.0)
    stream_context: bool = Field(False, description="reference streamed rung (not provided by this build)")
    context_row_chunk: int | None = Field(None, gt=0)
    adaptive_query_chunk: bool = Field(True, description="halve the query chunk on out-of-memory and retry")
    elements_budget: int | None = Field(None, gt=0, description="cap on context rows x features before subsampling")
    allow_subsample: bool = Field(True, description="subsample context rows (with a warning) when nothing fits")
    # resolved fields (filled by resolve())
    rung: str | None = None
    est_cache_gb: float | None = None
    resident_gb: float | None = None
    query_chunk: int | None = None
    dropped_context_rows: int = 0

    @field_validator("rung")
    @classmethod
    def _rung_known(cls, v):
        if v is not None and v not in RUNGS:
            raise ValueError(f"unknown rung {v!r}")
        return v

    @classmethod
    def coerce(cls, value) -> "MemoryPolicy":
        if value is None:
            return cls()
        if isinstance(value, MemoryPolicy):
            return value
        if isinstance(value, dict):
            return cls(**value)
        if isinstance(value, str):
            if value == "exact":
                return cls(allow_quantization=False)
            if value == "max_context":
                return cls(cache_dtype="int8")
            if value == "off":
                return cls(cache=False, reuse_context_cache=False)
            raise ValueError(f"unknown memory preset {value!r}; expected one of {MEMORY_PRESETS}")
        raise TypeError(f"memory policy must be a preset name, dict, MemoryPolicy or None, not {type(value).__name__}")

    def budget_gb(self, device_total_gb: float) -> float:
        if self.gpu_budget_absolute_gb is not None:
            return float(self.gpu_budget_absolute_gb)
        return self.gpu_budget_frac * device_total_gb

    def resolve(self, *, n_context_rows: int, n_groups: int, nlayers: int, embed_dim: int, head_dim: int,
                device_total_gb: float, n_gpus: int = 1) -> "MemoryPolicy":
        """Return a copy with ``rung`` / ``est_cache_gb`` / ``resident_gb`` /
        ``dropped_context_rows`` filled for this table."""
        if self.offload_to_host or self.stream_context:
            raise NotImplementedError("host-offload and streamed cache rungs are not provided by this build; use "
                                      "int8 or the multi-GPU context-sharded rung")
        bf16 = estimate_cache_gb(n_context_rows=n_context_rows, n_groups=n_groups, nlayers=nlayers,
                                 embed_dim=embed_dim)
        i8 = int8_footprint_gb(bf16, head_dim=head_dim)
        budget = self.budget_gb(device_total_gb)
        upd = {"est_cache_gb": bf16, "dropped_context_rows": 0}
        if not self.cache:
            upd.update(rung="no_cache", resident_gb=0.0)
        elif self.cache_dtype == "bf16" and bf16 <= budget:
            upd.update(rung="resident_bf16", resident_gb=bf16)
        elif (self.cache_dtype == "int8" or self.allow_quantization) and i8 <= budget:
            upd.update(rung="resident_int8", resident_gb=i8)
        elif n_gpus > 1 and (self.cache_dtype == "int8" or self.allow_quantization) and i8 / n_gpus <= budget:
            upd.update(rung="context_sharded_int8", resident_gb=i8 / n_gpus)
        elif self.allow_subsample:
            per_row = (i8 if (self.cache_dtype == "int8" or self.allow_quantization) else bf16) / max(n_context_rows, 1)
            keep = int(budget / per_row) if per_row > 0 else n_context_rows
            keep = max(1, min(keep, n_context_rows))
            upd.update(rung="subsample", resident_gb=per_row * keep, dropped_context_rows=n_context_rows - keep)
        else:
            raise MemoryError(f"context cache needs {i8:.1f} GiB even as int8 (budget {budget:.1f} GiB) and "
                              "subsampling is disabled")
        return self.model_copy(update=upd)

    def describe(self) -> dict:
        return self.model_dump()
