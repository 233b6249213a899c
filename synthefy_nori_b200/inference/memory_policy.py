"""Memory policy for the context cache (reference ``inference/memory_policy.py``).

The context K/V cache - not the model - is what exhausts GPU memory on large tables
(``L * (G+1) * N * 2 * E`` elements, reference ``memory_policy.py:368-389``).
``MemoryPolicy`` is the user-facing contract: the same field names, presets
(``"exact"``, ``"max_context"``, ``"off"``) and coercion rules (``None`` / preset name /
dict / instance) as the reference, so configurations carry over. ``resolve`` picks the
rung for a given table and device:

    no_cache -> resident_bf16 -> resident_int8 -> context_sharded_int8 -> subsample

    no_cache -> resident_bf16 -> resident_int8 -> context_sharded_int8 (several GPUs)
             -> offload_bf16 -> offload_int8 -> subsample   (stream_bf16 / stream_int8
                                                             when stream_context=True)

``offload_*``: the cache lives in pinned host RAM and each layer is copied in just before
it runs, the next layer's copy overlapping the current layer (``offload_to_host`` is a
permission, on by default; the host budget is a share of the RAM the process may really
use: the smaller of the kernel's available memory and the container's cgroup limit).
``stream_*`` (explicit ``stream_context=True``): the cache lives on the host in blocks of
``context_row_chunk`` context rows and the device never holds a full layer; query
attention merges the block partials by their log-sum-exps.  ``context_sharded_int8`` is
this build's multi-GPU rung (the cache split by context rows over the GPUs of one node,
``parallel/context_parallel.py``).  ``escalated`` records a rung the caller moved to after
an out-of-memory error (reference ``MemoryPolicy.escalated``).
"""

from __future__ import annotations

from typing import Literal

from pydantic import BaseModel, ConfigDict, Field, field_validator

CacheDtype = Literal["bf16", "int8"]
MEMORY_PRESETS = ("exact", "max_context", "off")
RUNGS = ("no_cache", "resident_bf16", "resident_int8", "offload_bf16", "offload_int8", "stream_bf16", "stream_int8",
         "context_sharded_int8", "context_row_chunk", "subsample", "plain_loop")
STREAM_RUNGS = ("stream_bf16", "stream_int8")
OFFLOAD_RUNGS = ("offload_bf16", "offload_int8")
KV_TENSORS_PER_ROW = 2
BYTES_PER_GIB = 1024 ** 3
CGROUP_LIMIT_FILES = ("/sys/fs/cgroup/memory.max", "/sys/fs/cgroup/memory/memory.limit_in_bytes")


def _cgroup_limit_gb(files=CGROUP_LIMIT_FILES) -> float | None:
    for f in files:
        try:
            raw = open(f).read().strip()
        except OSError:
            continue
        if raw in ("max", "") or not raw.isdigit():
            return None
        v = int(raw)
        return None if v >= 1 << 60 else v / BYTES_PER_GIB  # v1 reports a huge number for "no limit"
    return None


def host_memory_gb(meminfo: str = "/proc/meminfo", cgroup_files=CGROUP_LIMIT_FILES) -> float:
    """RAM this process may use: min(MemAvailable, cgroup limit) in GiB (0 if unknown)."""
    avail = None
    try:
        for line in open(meminfo):
            if line.startswith("MemAvailable:"):
                avail = int(line.split()[1]) * 1024 / BYTES_PER_GIB
                break
    except OSError:
        pass
    lim = _cgroup_limit_gb(cgroup_files)
    vals = [v for v in (avail, lim) if v is not None]
    return min(vals) if vals else 0.0


def default_stream_row_chunk(device_total_gb: float | None) -> int:
    """Context rows staged per streamed block when none is given (by device memory)."""
    v = 24.0 if device_total_gb is None else device_total_gb
    return 16384 if v >= 80 else (8192 if v >= 40 else 2048)


def estimate_cache_gb(*, n_context_rows: int, n_groups: int, nlayers: int, embed_dim: int,
                      bytes_per_element: int = 2) -> float:
    """Context cache footprint in GiB (``n_groups`` counts the target token too)."""
    return nlayers * n_groups * n_context_rows * KV_TENSORS_PER_ROW * embed_dim * bytes_per_element / BYTES_PER_GIB


def int8_footprint_gb(est_bf16_gb: float, *, head_dim: int) -> float:
    """The same cache stored int8 with one fp32 scale per (token, head) vector."""
    return est_bf16_gb / 2.0 * (1.0 + 4.0 / max(head_dim, 1))


class ContextTooLargeError(RuntimeError, MemoryError):
    """The context cannot fit without a fallback the caller's policy forbids (subsampling
    disabled). A caller condition, not a device fault; the message names the setting to change.
    Also a ``MemoryError``, so handlers written for the memory ladder catch it."""


class MemoryPolicy(BaseModel):
    """How ``predict`` may spend GPU memory on the context cache."""

    model_config = ConfigDict(extra="forbid", frozen=True)

    cache: bool = Field(True, description="build a context K/V cache (False: recompute the context per query chunk)")
    reuse_context_cache: bool = Field(True, description="keep the cache across predict calls with the same context")
    cache_dtype: CacheDtype = Field("bf16", description="starting precision of the cache")
    allow_quantization: bool = Field(True, description="may fall back from bf16 to int8 when bf16 does not fit")
    gpu_budget_frac: float = Field(0.6, gt=0.0, le=1.0, description="fraction of device memory the cache may use")
    gpu_budget_absolute_gb: float | None = Field(None, gt=0.0)
    offload_to_host: bool = Field(True, description="may the cache live in host RAM (one layer copied in at a "
                                                    "time) when it cannot stay resident")
    host_budget_frac: float = Field(0.5, gt=0.0, le=1.0, description="share of usable host RAM for an offloaded cache")
    host_budget_absolute_gb: float | None = Field(None, ge=0.0, description="hard host ceiling (0 = never offload)")
    stream_context: bool = Field(False, description="keep the cache on the host in row blocks; the device never "
                                                    "holds a full layer")
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

    def host_budget(self, host_total_gb: float | None = None) -> float:
        if self.host_budget_absolute_gb is not None:
            return float(self.host_budget_absolute_gb)
        return self.host_budget_frac * (host_memory_gb() if host_total_gb is None else host_total_gb)

    def resolve(self, *, n_context_rows: int, n_groups: int, nlayers: int, embed_dim: int, head_dim: int,
                device_total_gb: float, n_gpus: int = 1, host_total_gb: float | None = None) -> "MemoryPolicy":
        """Return a copy with ``rung`` / ``est_cache_gb`` / ``resident_gb`` /
        ``dropped_context_rows`` (and the streamed ``context_row_chunk``) filled for this
        table."""
        if self.stream_context and not self.cache:
            raise ValueError("stream_context=True requires cache=True")
        if self.stream_context and not self.offload_to_host:
            raise ValueError("stream_context=True requires offload_to_host=True (the stream lives in host RAM)")
        bf16 = estimate_cache_gb(n_context_rows=n_context_rows, n_groups=n_groups, nlayers=nlayers,
                                 embed_dim=embed_dim)
        i8 = int8_footprint_gb(bf16, head_dim=head_dim)
        q_ok = self.cache_dtype == "int8" or self.allow_quantization
        budget = self.budget_gb(device_total_gb)
        upd = {"est_cache_gb": bf16, "dropped_context_rows": 0}
        per_layer = bf16 / max(nlayers, 1)
        if not self.cache:
            upd.update(rung="no_cache", resident_gb=0.0)
        elif self.stream_context:
            chunk = self.context_row_chunk or default_stream_row_chunk(device_total_gb)
            use_i8 = self.cache_dtype == "int8"
            host = self.host_budget(host_total_gb)
            size = i8 if use_i8 else bf16
            if size > host:
                if not q_ok or use_i8 or i8 > host:
                    raise ContextTooLargeError(f"streamed cache needs {size:.1f} GiB of host RAM (budget {host:.1f} GiB): "
                                               "raise host_budget_absolute_gb / host_budget_frac or use an int8 cache")
                use_i8, size = True, i8
            upd.update(rung="stream_int8" if use_i8 else "stream_bf16", context_row_chunk=int(chunk),
                       resident_gb=2 * per_layer * min(1.0, chunk / max(n_context_rows, 1)),
                       reuse_context_cache=False)
        elif self.cache_dtype == "bf16" and bf16 <= budget:
            upd.update(rung="resident_bf16", resident_gb=bf16)
        elif q_ok and i8 <= budget:
            upd.update(rung="resident_int8", resident_gb=i8)
        elif n_gpus > 1 and q_ok and i8 / n_gpus <= budget:  # NVLink beats the host link
            upd.update(rung="context_sharded_int8", resident_gb=i8 / n_gpus)
        elif self.offload_to_host and self.cache_dtype == "bf16" and bf16 <= self.host_budget(host_total_gb) \
                and 2 * per_layer <= budget:
            upd.update(rung="offload_bf16", resident_gb=2 * per_layer)
        elif self.offload_to_host and q_ok and i8 <= self.host_budget(host_total_gb) \
                and 2 * per_layer * i8 / max(bf16, 1e-12) <= budget:
            upd.update(rung="offload_int8", resident_gb=2 * per_layer * i8 / max(bf16, 1e-12))
        elif self.allow_subsample:
            per_row = (i8 if q_ok else bf16) / max(n_context_rows, 1)
            keep = int(budget / per_row) if per_row > 0 else n_context_rows
            keep = max(1, min(keep, n_context_rows))
            upd.update(rung="subsample", resident_gb=per_row * keep, dropped_context_rows=n_context_rows - keep)
        else:
            raise ContextTooLargeError(f"context cache needs {i8:.1f} GiB even as int8 (budget {budget:.1f} GiB) "
                                       "and subsampling is disabled: raise elements_budget / the device budget, or "
                                       "allow_subsample=True")
        return self.model_copy(update=upd)

    def next_rung(self) -> str | None:
        """The rung to try after an out-of-memory error on the current one."""
        order = {"resident_bf16": "resident_int8" if self.allow_quantization else "offload_bf16",
                 "resident_int8": "offload_int8", "offload_bf16": "offload_int8", "offload_int8": "stream_int8",
                 "stream_bf16": "stream_int8", "stream_int8": None, "context_sharded_int8": "stream_int8",
                 "no_cache": None, "subsample": None, "plain_loop": None, "context_row_chunk": "plain_loop"}
        nxt = order.get(self.rung or "", None)
        if nxt is not None and nxt.startswith(("offload", "stream")) and not self.offload_to_host:
            return "plain_loop"
        return nxt

    def escalated(self, rung: str, *, context_row_chunk: int | None = None, dropped_context_rows: int | None = None,
                  query_chunk: int | None = None) -> "MemoryPolicy":
        """A copy recording an escalation the caller made after an out-of-memory error."""
        if rung not in RUNGS:
            raise ValueError(f"unknown rung {rung!r}")
        if self.stream_context and rung not in STREAM_RUNGS:
            raise ValueError(f"stream_context=True cannot escalate to {rung!r}: it stays on a streamed rung")
        upd: dict = {"rung": rung}
        if context_row_chunk is not None:
            upd["context_row_chunk"] = int(context_row_chunk)
        if dropped_context_rows is not None:
            upd["dropped_context_rows"] = int(dropped_context_rows)
        if query_chunk is not None:
            upd["query_chunk"] = int(query_chunk)
        if rung == "plain_loop":
            upd.update(cache=False, reuse_context_cache=False, offload_to_host=False)
        if rung in STREAM_RUNGS and not self.context_row_chunk and context_row_chunk is None:
            upd["context_row_chunk"] = 4096
        return self.model_copy(update=upd)

    def placement(self) -> tuple[str, str, int | None]:
        """(cache dtype, placement, stream block rows) of the resolved rung."""
        r = self.rung or "resident_bf16"
        dtype = "int8" if (r.endswith("int8") or self.cache_dtype == "int8") else "bf16"
        if r in OFFLOAD_RUNGS:
            return dtype, "offload", None
        if r in STREAM_RUNGS:
            return dtype, "stream", self.context_row_chunk or 4096
        return dtype, "resident", None

    def describe(self) -> dict:
        return self.model_dump()
