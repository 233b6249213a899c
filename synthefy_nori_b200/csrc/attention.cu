// Flash attention forward / backward for the two attention families of the Nori
// encoder, reading and writing the framework's own layouts directly (no transposes):
//
//   * sequence (ICL) attention per (table, column, head) over context rows
//     (reference model/layer.py:1407-1441: context self-attention and query->context
//     cross-attention), Q/K/V head-major [.., H, rows, 64] written by the projection
//     GEMM's head-major epilogue;
//   * feature (within-row) attention per (table row, head) over the G+1 tokens of a
//     row (reference model/layer.py:1391-1405).
//
// Head dim is padded to 64 in the inputs (padding columns are zero). Outputs go to a
// generic 3-level strided layout, typically token-major [tokens, H * D] so the output
// projection GEMM reads them as its A operand.
//
// Tiles: 64 query rows per CTA (4 warps x 16 rows), 64-key K/V tiles double-buffered
// in shared memory with an XOR swizzle; QK^T and PV on mma.m16n8k16 bf16 with fp32
// accumulation, online softmax in registers (exp2 with folded log2 e), natural-log LSE
// saved for the backward pass and for partial-softmax merges.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "sm100.cuh"
#include "tma_host.h"

namespace nori {

// bh -> (i0, i1, i2) with i2 fastest: i2 = bh % d2, i1 = (bh / d2) % d1, i0 = bh / (d1 d2)
struct Layout3 {
  int64_t s0, s1, s2, row;
  int d1, d2;
  // bh < 2^31 (grids and BH are int): 32-bit division, much cheaper on the GPU than 64-bit
  __host__ __device__ int64_t offset(int64_t bh, int64_t r) const {
    const int b = static_cast<int>(bh);
    const int i2 = b % d2;
    const int t = b / d2;
    const int i1 = t % d1;
    const int i0 = t / d1;
    return static_cast<int64_t>(i0) * s0 + static_cast<int64_t>(i1) * s1 + static_cast<int64_t>(i2) * s2 + r * row;
  }
};

constexpr int kD = 64;      // padded head dim
constexpr int kBlkQ = 64;   // query rows per CTA
constexpr int kBlkK = 64;   // keys per tile
constexpr int kAttnThreads = 128;

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Swizzled byte offset of (row, 16-byte chunk) in a [rows][64 bf16] tile.
__device__ __forceinline__ int swz(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

// Load a [64 rows][64 cols] bf16 tile; rows >= n_valid and columns >= d_valid read as 0.
__device__ __forceinline__ void load_tile(uint8_t* tile, const __nv_bfloat16* base, int64_t row_stride, int row0,
                                          int n_valid, int d_valid, int tid, int nthreads) {
  for (int i = tid; i < 64 * 8; i += nthreads) {
    const int r = i >> 3, c = i & 7;
    const int gr = row0 + r;
    int bytes = 0;
    const __nv_bfloat16* src = base;
    if (gr < n_valid) {
      const int rem = d_valid - c * 8;
      bytes = rem >= 8 ? 16 : (rem > 0 ? rem * 2 : 0);
      if (bytes > 0) src = base + static_cast<int64_t>(gr) * row_stride + c * 8;
    }
    cp_async16(tile + swz(r, c), src, bytes);
  }
}

// ---------------------------------------------------------------- forward
struct AttnFwdParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  __nv_bfloat16* o;
  float* lse;  // [BH, Nq] or null
  Layout3 lq, lk, lv, lo;
  int BH, Nq, Nk, d_valid;  // d_valid: true head dim (<= 64) of the output
  int n_tiles_q;
  int q_d_valid;            // columns of Q / K / V to read (<= 64)
  float scale_log2;         // softmax scale * log2(e)
};

// Per-warp running state of the forward pass (16 query rows per warp).
struct FwdState {
  uint32_t qf[4][4];
  float o[8][4];
  float m0, m1, l0, l1;
};

__device__ __forceinline__ void fwd_init(FwdState& st, const uint8_t* sq, int warp, int lane) {
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const int r = warp * 16 + (lane & 15);
    const int c = kk * 2 + (lane >> 4);
    ldsm_x4(st.qf[kk], smem_u32(sq + swz(r, c)));
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) st.o[i][0] = st.o[i][1] = st.o[i][2] = st.o[i][3] = 0.f;
  st.m0 = st.m1 = -INFINITY;
  st.l0 = st.l1 = 0.f;
}

// One 64-key tile: S = Q K^T, online softmax, O += P V.
__device__ __forceinline__ void fwd_tile(FwdState& st, const uint8_t* sk, const uint8_t* sv, int kbase, int Nk,
                                         float scale_log2, int lane) {
  float s[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
    for (int j2 = 0; j2 < 4; ++j2) {
      // two key n-tiles (16 keys) x 16 d: (keys 0-7, d lo), (keys 0-7, d hi), (keys 8-15, d lo), (8-15, d hi)
      uint32_t b[4];
      const int key = j2 * 16 + (lane & 7) + ((lane >> 4) << 3);
      const int c = kk * 2 + ((lane >> 3) & 1);
      ldsm_x4(b, smem_u32(sk + swz(key, c)));
      mma16816(s[2 * j2], st.qf[kk], b[0], b[1]);
      mma16816(s[2 * j2 + 1], st.qf[kk], b[2], b[3]);
    }
  }
  if (kbase + kBlkK > Nk) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c0 = kbase + j * 8 + (lane & 3) * 2;
      if (c0 >= Nk) s[j][0] = s[j][2] = -INFINITY;
      if (c0 + 1 >= Nk) s[j][1] = s[j][3] = -INFINITY;
    }
  }
  float mx0 = st.m0, mx1 = st.m1;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]) * scale_log2);
    mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]) * scale_log2);
  }
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
  }
  const float a0 = (st.m0 == -INFINITY) ? 0.f : exp2f(st.m0 - mx0);
  const float a1 = (st.m1 == -INFINITY) ? 0.f : exp2f(st.m1 - mx1);
  const float mb0 = (mx0 == -INFINITY) ? 0.f : mx0;
  const float mb1 = (mx1 == -INFINITY) ? 0.f : mx1;
  st.m0 = mx0;
  st.m1 = mx1;
  float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    s[j][0] = exp2f(s[j][0] * scale_log2 - mb0);
    s[j][1] = exp2f(s[j][1] * scale_log2 - mb0);
    s[j][2] = exp2f(s[j][2] * scale_log2 - mb1);
    s[j][3] = exp2f(s[j][3] * scale_log2 - mb1);
    rs0 += s[j][0] + s[j][1];
    rs1 += s[j][2] + s[j][3];
  }
  st.l0 = st.l0 * a0 + rs0;
  st.l1 = st.l1 * a1 + rs1;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    st.o[i][0] *= a0;
    st.o[i][1] *= a0;
    st.o[i][2] *= a1;
    st.o[i][3] *= a1;
  }
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    uint32_t pa[4];
    pa[0] = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
    pa[1] = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
    pa[2] = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
    pa[3] = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
    for (int i2 = 0; i2 < 4; ++i2) {
      uint32_t b[4];
      const int key = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
      const int c = i2 * 2 + (lane >> 4);
      ldsm_x4_t(b, smem_u32(sv + swz(key, c)));
      mma16816(st.o[2 * i2], pa, b[0], b[1]);
      mma16816(st.o[2 * i2 + 1], pa, b[2], b[3]);
    }
  }
}

__device__ __forceinline__ void fwd_store(FwdState& st, __nv_bfloat16* ob, int64_t row_stride, float* lse, int64_t bh,
                                          int q0, int Nq, int d_valid, int warp, int lane) {
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    st.l0 += __shfl_xor_sync(0xffffffffu, st.l0, off);
    st.l1 += __shfl_xor_sync(0xffffffffu, st.l1, off);
  }
  const float inv0 = st.l0 > 0.f ? 1.f / st.l0 : 0.f;
  const float inv1 = st.l1 > 0.f ? 1.f / st.l1 : 0.f;
  const int r0 = q0 + warp * 16 + (lane >> 2);
  const int r1 = r0 + 8;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = i * 8 + (lane & 3) * 2;
    if (c < d_valid) {
      if (r0 < Nq)
        *reinterpret_cast<uint32_t*>(ob + static_cast<int64_t>(r0) * row_stride + c) =
            pack_bf16x2(st.o[i][0] * inv0, st.o[i][1] * inv0);
      if (r1 < Nq)
        *reinterpret_cast<uint32_t*>(ob + static_cast<int64_t>(r1) * row_stride + c) =
            pack_bf16x2(st.o[i][2] * inv1, st.o[i][3] * inv1);
    }
  }
  if (lse != nullptr && (lane & 3) == 0) {
    constexpr float kLn2 = 0.6931471805599453f;
    if (r0 < Nq) lse[bh * Nq + r0] = st.l0 > 0.f ? (st.m0 + log2f(st.l0)) * kLn2 : -INFINITY;
    if (r1 < Nq) lse[bh * Nq + r1] = st.l1 > 0.f ? (st.m1 + log2f(st.l1)) * kLn2 : -INFINITY;
  }
}

// KV_BUF = 2: K / V tiles double-buffered across the key loop; KV_BUF = 1: the whole key
// sequence is one tile (short sequences such as the within-row feature attention), so a
// CTA needs 24 KB instead of 40 KB of shared memory and more CTAs share an SM.
template <int KV_BUF>
__global__ void __launch_bounds__(kAttnThreads) attn_fwd_kernel(AttnFwdParams p) {
  __shared__ __align__(128) uint8_t sq[kBlkQ * 128];
  __shared__ __align__(128) uint8_t sk[KV_BUF][kBlkK * 128];
  __shared__ __align__(128) uint8_t sv[KV_BUF][kBlkK * 128];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t bh = blockIdx.x / p.n_tiles_q;
  const int q0 = static_cast<int>(blockIdx.x % p.n_tiles_q) * kBlkQ;
  const __nv_bfloat16* qb = p.q + p.lq.offset(bh, 0);
  const __nv_bfloat16* kb = p.k + p.lk.offset(bh, 0);
  const __nv_bfloat16* vb = p.v + p.lv.offset(bh, 0);

  load_tile(sq, qb, p.lq.row, q0, p.Nq, p.q_d_valid, tid, kAttnThreads);
  load_tile(sk[0], kb, p.lk.row, 0, p.Nk, p.q_d_valid, tid, kAttnThreads);
  load_tile(sv[0], vb, p.lv.row, 0, p.Nk, p.q_d_valid, tid, kAttnThreads);
  cp_async_commit();

  FwdState st;
  if constexpr (KV_BUF == 1) {
    cp_async_wait<0>();
    __syncthreads();
    fwd_init(st, sq, warp, lane);
    fwd_tile(st, sk[0], sv[0], 0, p.Nk, p.scale_log2, lane);
  } else {
    const int n_tiles = (p.Nk + kBlkK - 1) / kBlkK;
    for (int t = 0; t < n_tiles; ++t) {
      const int buf = t & 1;
      if (t + 1 < n_tiles) {
        load_tile(sk[buf ^ 1], kb, p.lk.row, (t + 1) * kBlkK, p.Nk, p.q_d_valid, tid, kAttnThreads);
        load_tile(sv[buf ^ 1], vb, p.lv.row, (t + 1) * kBlkK, p.Nk, p.q_d_valid, tid, kAttnThreads);
      }
      cp_async_commit();
      cp_async_wait<1>();
      __syncthreads();
      if (t == 0) fwd_init(st, sq, warp, lane);
      fwd_tile(st, sk[buf], sv[buf], t * kBlkK, p.Nk, p.scale_log2, lane);
      __syncthreads();
    }
  }
  fwd_store(st, p.o + p.lo.offset(bh, 0), p.lo.row, p.lse, bh, q0, p.Nq, p.d_valid, warp, lane);
}

// ---------------------------------------------------------------- int8 K/V forward
// K / V stored int8 with one fp32 scale per (row, head); tiles are dequantized on the
// way into shared memory (each thread: 8 int8 -> 8 bf16), so no bf16 copy of the
// cache exists in global memory.
struct AttnQ8Params {
  const __nv_bfloat16* q;
  const int8_t* k;
  const int8_t* v;
  const float* ks;
  const float* vs;
  __nv_bfloat16* o;
  float* lse;
  Layout3 lq, lkv, ls, lo;
  int BH, Nq, Nk, d_valid;
  int n_tiles_q;
  float scale_log2;
};

__device__ __forceinline__ void load_tile_q8(uint8_t* tile, const int8_t* base, const float* sbase, int64_t row_stride,
                                             int64_t srow, int row0, int n_valid, int d_valid, int tid, int nthreads) {
  for (int i = tid; i < 64 * 8; i += nthreads) {
    const int r = i >> 3, c = i & 7;
    const int gr = row0 + r;
    uint4 w = make_uint4(0u, 0u, 0u, 0u);
    if (gr < n_valid && c * 8 < d_valid) {
      const uint2 raw = *reinterpret_cast<const uint2*>(base + static_cast<int64_t>(gr) * row_stride + c * 8);
      const float sc = sbase[static_cast<int64_t>(gr) * srow];
      const uint32_t lo = raw.x, hi = raw.y;
      auto cvt = [&](uint32_t word, int byte) -> float {
        return static_cast<float>(static_cast<int8_t>((word >> (8 * byte)) & 0xFFu)) * sc;
      };
      w.x = pack_bf16x2(cvt(lo, 0), cvt(lo, 1));
      w.y = pack_bf16x2(cvt(lo, 2), cvt(lo, 3));
      w.z = pack_bf16x2(cvt(hi, 0), cvt(hi, 1));
      w.w = pack_bf16x2(cvt(hi, 2), cvt(hi, 3));
    }
    *reinterpret_cast<uint4*>(tile + swz(r, c)) = w;
  }
}

// Register-staged int8 tile loads: fetch the next tile's raw bytes and scales while the
// current tile computes, then dequantise into shared memory (4 chunks of 8 values per
// thread per tile with 128 threads).
struct Q8Stage {
  uint2 raw[4];
  float sc[4];
};

__device__ __forceinline__ void q8_fetch(Q8Stage& st, const int8_t* base, const float* sbase, int64_t row_stride,
                                         int64_t srow, int row0, int n_valid, int d_valid, int tid) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = tid + k * kAttnThreads;
    const int r = i >> 3, c = i & 7;
    const int gr = row0 + r;
    if (gr < n_valid && c * 8 < d_valid) {
      st.raw[k] = *reinterpret_cast<const uint2*>(base + static_cast<int64_t>(gr) * row_stride + c * 8);
      st.sc[k] = sbase[static_cast<int64_t>(gr) * srow];
    } else {
      st.raw[k] = make_uint2(0u, 0u);
      st.sc[k] = 0.f;
    }
  }
}

__device__ __forceinline__ void q8_commit(const Q8Stage& st, uint8_t* tile, int tid) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = tid + k * kAttnThreads;
    const int r = i >> 3, c = i & 7;
    const uint32_t lo = st.raw[k].x, hi = st.raw[k].y;
    const float sc = st.sc[k];
    auto cvt = [&](uint32_t word, int byte) -> float {
      return static_cast<float>(static_cast<int8_t>((word >> (8 * byte)) & 0xFFu)) * sc;
    };
    *reinterpret_cast<uint4*>(tile + swz(r, c)) =
        make_uint4(pack_bf16x2(cvt(lo, 0), cvt(lo, 1)), pack_bf16x2(cvt(lo, 2), cvt(lo, 3)),
                   pack_bf16x2(cvt(hi, 0), cvt(hi, 1)), pack_bf16x2(cvt(hi, 2), cvt(hi, 3)));
  }
}

__global__ void __launch_bounds__(kAttnThreads) attn_fwd_q8_kernel(AttnQ8Params p) {
  __shared__ __align__(128) uint8_t sq[kBlkQ * 128];
  __shared__ __align__(128) uint8_t sk[kBlkK * 128];
  __shared__ __align__(128) uint8_t sv[kBlkK * 128];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t bh = blockIdx.x / p.n_tiles_q;
  const int q0 = static_cast<int>(blockIdx.x % p.n_tiles_q) * kBlkQ;
  const __nv_bfloat16* qb = p.q + p.lq.offset(bh, 0);
  const int8_t* kb = p.k + p.lkv.offset(bh, 0);
  const int8_t* vb = p.v + p.lkv.offset(bh, 0);
  const float* ksb = p.ks + p.ls.offset(bh, 0);
  const float* vsb = p.vs + p.ls.offset(bh, 0);
  load_tile(sq, qb, p.lq.row, q0, p.Nq, p.d_valid, tid, kAttnThreads);
  cp_async_commit();
  cp_async_wait<0>();
  const int n_tiles = (p.Nk + kBlkK - 1) / kBlkK;
  FwdState st;
  for (int t = 0; t < n_tiles; ++t) {
    load_tile_q8(sk, kb, ksb, p.lkv.row, p.ls.row, t * kBlkK, p.Nk, p.d_valid, tid, kAttnThreads);
    load_tile_q8(sv, vb, vsb, p.lkv.row, p.ls.row, t * kBlkK, p.Nk, p.d_valid, tid, kAttnThreads);
    __syncthreads();
    if (t == 0) fwd_init(st, sq, warp, lane);
    fwd_tile(st, sk, sv, t * kBlkK, p.Nk, p.scale_log2, lane);
    __syncthreads();
  }
  fwd_store(st, p.o + p.lo.offset(bh, 0), p.lo.row, p.lse, bh, q0, p.Nq, p.d_valid, warp, lane);
}

// ---------------------------------------------------------------- backward
// Dvec[bh, i] = sum_d dO[i, d] * O[i, d]; one thread per (head, row), 16-byte loads.
__global__ void attn_bwd_dot_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                    Layout3 lo, Layout3 ldo, int BH, int Nq, int d_valid, float* __restrict__ dvec) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(BH) * Nq) return;
  const int64_t bh = idx / Nq;
  const int r = static_cast<int>(idx % Nq);
  const __nv_bfloat16* op = o + lo.offset(bh, r);
  const __nv_bfloat16* dp = dout + ldo.offset(bh, r);
  float s = 0.f;
  for (int c = 0; c < d_valid; c += 8) {
    const uint4 a = *reinterpret_cast<const uint4*>(op + c);
    const uint4 b = *reinterpret_cast<const uint4*>(dp + c);
    const uint32_t aa[4] = {a.x, a.y, a.z, a.w}, bb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) s += bf16lo(aa[i]) * bf16lo(bb[i]) + bf16hi(aa[i]) * bf16hi(bb[i]);
  }
  dvec[idx] = s;
}

struct AttnBwdParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  const __nv_bfloat16* dout;
  const __nv_bfloat16* o;  // forward output (read by the single-tile kernel for D = dO . O)
  const float* lse;
  const float* dvec;
  float* dq;  // fp32 accumulator addressed through ldq
  __nv_bfloat16* dq16;  // or, with a single key tile, dQ written once in bf16 through ldq
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  Layout3 lq, lk, lv, ldo, ldk, ldv, ldq, lo;
  int BH, Nq, Nk, d_valid, q_d_valid;
  int n_tiles_k;
  float scale, scale_log2;
};

// One (64-key, 64-query) tile of the backward: S^T = K Q^T and dP^T = V dO^T, P^T and
// dS^T, dV += P^T dO, dK += dS^T Q (both unscaled), dS^T through shared memory, and this
// warp's 16 rows of dQ = dS K (unscaled) into dqa. Ends with all warps past the dS^T
// stores (one __syncthreads inside).
__device__ __forceinline__ void bwd_tile(const uint8_t* sq, const uint8_t* sdo, const uint8_t* sk, uint8_t* sds,
                                         const float* slse, const float* sdv, const uint32_t (&kf)[4][4],
                                         const uint32_t (&vf)[4][4], int k0, int q0, int Nk, int Nq,
                                         float scale_log2, int warp, int lane, float (&dk)[8][4],
                                         float (&dv)[8][4], float (&dqa)[8][4]) {
    // S^T = K Q^T (16 keys x 64 q) and dP^T = V dO^T
    float st[8][4], dpt[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) st[j][e] = dpt[j][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int j2 = 0; j2 < 4; ++j2) {
        uint32_t b[4];
        const int qr = j2 * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = kk * 2 + ((lane >> 3) & 1);
        ldsm_x4(b, smem_u32(sq + swz(qr, c)));
        mma16816(st[2 * j2], kf[kk], b[0], b[1]);
        mma16816(st[2 * j2 + 1], kf[kk], b[2], b[3]);
        ldsm_x4(b, smem_u32(sdo + swz(qr, c)));
        mma16816(dpt[2 * j2], vf[kk], b[0], b[1]);
        mma16816(dpt[2 * j2 + 1], vf[kk], b[2], b[3]);
      }
    }
    // P^T and dS^T ; rows = keys (g, g+8 of the warp's 16), columns = queries
    const int key0 = k0 + warp * 16 + (lane >> 2);
    constexpr float kLog2e = 1.4426950408889634f;
    // packed to bf16 pairs at once ((e0, e1) and (e2, e3) of each 8-query tile), so the
    // fp32 tiles are dead before the dV / dK products
    uint32_t pp[8][2], dd[8][2];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float pv[4], ds[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qc = j * 8 + (lane & 3) * 2 + (e & 1);
        const int key = key0 + ((e >> 1) << 3);
        pv[e] = 0.f;
        if (key < Nk && q0 + qc < Nq) pv[e] = exp2f(st[j][e] * scale_log2 - slse[qc] * kLog2e);
        ds[e] = pv[e] * (dpt[j][e] - sdv[qc]);
      }
      pp[j][0] = pack_bf16x2(pv[0], pv[1]);
      pp[j][1] = pack_bf16x2(pv[2], pv[3]);
      dd[j][0] = pack_bf16x2(ds[0], ds[1]);
      dd[j][1] = pack_bf16x2(ds[2], ds[3]);
    }
    // dV += P^T dO ; dK += dS^T Q  (A from registers; B = dO / Q with trans loads)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t pa[4] = {pp[2 * kk][0], pp[2 * kk][1], pp[2 * kk + 1][0], pp[2 * kk + 1][1]};
      const uint32_t da[4] = {dd[2 * kk][0], dd[2 * kk][1], dd[2 * kk + 1][0], dd[2 * kk + 1][1]};
#pragma unroll
      for (int i2 = 0; i2 < 4; ++i2) {
        uint32_t b[4];
        const int qr = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int c = i2 * 2 + (lane >> 4);
        ldsm_x4_t(b, smem_u32(sdo + swz(qr, c)));
        mma16816(dv[2 * i2], pa, b[0], b[1]);
        mma16816(dv[2 * i2 + 1], pa, b[2], b[3]);
        ldsm_x4_t(b, smem_u32(sq + swz(qr, c)));
        mma16816(dk[2 * i2], da, b[0], b[1]);
        mma16816(dk[2 * i2 + 1], da, b[2], b[3]);
      }
    }
    // dS^T -> shared (bf16, [key][q]) for the dQ product
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int qc = j * 8 + (lane & 3) * 2;
      const int kr = warp * 16 + (lane >> 2);
      *reinterpret_cast<uint32_t*>(sds + swz(kr, qc >> 3) + (qc & 7) * 2) = dd[j][0];
      *reinterpret_cast<uint32_t*>(sds + swz(kr + 8, qc >> 3) + (qc & 7) * 2) = dd[j][1];
    }
    __syncthreads();
    // dQ[q rows warp*16..] += dS (q x keys) K (keys x d) * scale ; A = dS via trans load of dS^T
    {
#pragma unroll
      for (int i = 0; i < 8; ++i) dqa[i][0] = dqa[i][1] = dqa[i][2] = dqa[i][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t a[4];
        // A[q][key] = dS^T[key][q]: matrices (q 0-7,key 0-7),(q 8-15,key 0-7),(q 0-7,key 8-15),(q 8-15,key 8-15)
        {
          const int key = kk * 16 + (lane & 7) + ((lane >> 4) << 3);
          const int qcol = warp * 16 + (((lane >> 3) & 1) << 3);
          ldsm_x4_t(a, smem_u32(sds + swz(key, qcol >> 3)));
        }
#pragma unroll
        for (int i2 = 0; i2 < 4; ++i2) {
          uint32_t b[4];
          const int key = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
          const int c = i2 * 2 + (lane >> 4);
          ldsm_x4_t(b, smem_u32(sk + swz(key, c)));
          mma16816(dqa[2 * i2], a, b[0], b[1]);
          mma16816(dqa[2 * i2 + 1], a, b[2], b[3]);
        }
      }
    }
}

__global__ void __launch_bounds__(kAttnThreads) attn_bwd_kernel(AttnBwdParams p) {
  __shared__ __align__(128) uint8_t sk[kBlkK * 128];
  __shared__ __align__(128) uint8_t sv[kBlkK * 128];
  __shared__ __align__(128) uint8_t sq[kBlkQ * 128];
  __shared__ __align__(128) uint8_t sdo[kBlkQ * 128];
  __shared__ __align__(128) uint8_t sds[kBlkK * 128];  // dS^T [key][q]
  __shared__ float slse[kBlkQ], sdv[kBlkQ];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t bh = blockIdx.x / p.n_tiles_k;
  const int k0 = static_cast<int>(blockIdx.x % p.n_tiles_k) * kBlkK;
  const __nv_bfloat16* qb = p.q + p.lq.offset(bh, 0);
  const __nv_bfloat16* kb = p.k + p.lk.offset(bh, 0);
  const __nv_bfloat16* vb = p.v + p.lv.offset(bh, 0);
  const __nv_bfloat16* dob = p.dout + p.ldo.offset(bh, 0);

  load_tile(sk, kb, p.lk.row, k0, p.Nk, p.q_d_valid, tid, kAttnThreads);
  load_tile(sv, vb, p.lv.row, k0, p.Nk, p.q_d_valid, tid, kAttnThreads);
  cp_async_commit();

  float dk[8][4], dv[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;

  uint32_t kf[4][4], vf[4][4];
  const int n_qt = (p.Nq + kBlkQ - 1) / kBlkQ;
  for (int qt = 0; qt < n_qt; ++qt) {
    const int q0 = qt * kBlkQ;
    load_tile(sq, qb, p.lq.row, q0, p.Nq, p.q_d_valid, tid, kAttnThreads);
    load_tile(sdo, dob, p.ldo.row, q0, p.Nq, p.d_valid, tid, kAttnThreads);
    cp_async_commit();
    if (tid < kBlkQ) {
      const int r = q0 + tid;
      slse[tid] = r < p.Nq ? p.lse[bh * p.Nq + r] : INFINITY;
      sdv[tid] = r < p.Nq ? p.dvec[bh * p.Nq + r] : 0.f;
    }
    cp_async_wait<0>();
    __syncthreads();
    if (qt == 0) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int r = warp * 16 + (lane & 15);
        const int c = kk * 2 + (lane >> 4);
        ldsm_x4(kf[kk], smem_u32(sk + swz(r, c)));
        ldsm_x4(vf[kk], smem_u32(sv + swz(r, c)));
      }
    }
    float dqa[8][4];
    bwd_tile(sq, sdo, sk, sds, slse, sdv, kf, vf, k0, q0, p.Nk, p.Nq, p.scale_log2, warp, lane, dk, dv, dqa);
    {
      const int r0 = q0 + warp * 16 + (lane >> 2);
      if (p.dq16 != nullptr) {  // single key tile: this CTA owns these dQ rows outright
        __nv_bfloat16* dqh = p.dq16 + p.ldq.offset(bh, 0);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int c = i * 8 + (lane & 3) * 2;
          if (c >= p.d_valid) continue;
          if (r0 < p.Nq)
            *reinterpret_cast<uint32_t*>(dqh + static_cast<int64_t>(r0) * p.ldq.row + c) =
                pack_bf16x2(dqa[i][0] * p.scale, dqa[i][1] * p.scale);
          if (r0 + 8 < p.Nq)
            *reinterpret_cast<uint32_t*>(dqh + static_cast<int64_t>(r0 + 8) * p.ldq.row + c) =
                pack_bf16x2(dqa[i][2] * p.scale, dqa[i][3] * p.scale);
        }
        __syncthreads();
        continue;
      }
      float* dqb = p.dq + p.ldq.offset(bh, 0);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c = i * 8 + (lane & 3) * 2;
        if (c >= p.d_valid) continue;
        if (r0 < p.Nq) {
          atomicAdd(dqb + static_cast<int64_t>(r0) * p.ldq.row + c, dqa[i][0] * p.scale);
          atomicAdd(dqb + static_cast<int64_t>(r0) * p.ldq.row + c + 1, dqa[i][1] * p.scale);
        }
        if (r0 + 8 < p.Nq) {
          atomicAdd(dqb + static_cast<int64_t>(r0 + 8) * p.ldq.row + c, dqa[i][2] * p.scale);
          atomicAdd(dqb + static_cast<int64_t>(r0 + 8) * p.ldq.row + c + 1, dqa[i][3] * p.scale);
        }
      }
    }
    __syncthreads();
  }
  // write dK (scaled), dV
  const int r0 = k0 + warp * 16 + (lane >> 2);
  __nv_bfloat16* dkb = p.dk + p.ldk.offset(bh, 0);
  __nv_bfloat16* dvb = p.dv + p.ldv.offset(bh, 0);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = i * 8 + (lane & 3) * 2;
    if (c >= p.d_valid) continue;
    if (r0 < p.Nk) {
      *reinterpret_cast<uint32_t*>(dkb + static_cast<int64_t>(r0) * p.ldk.row + c) =
          pack_bf16x2(dk[i][0] * p.scale, dk[i][1] * p.scale);
      *reinterpret_cast<uint32_t*>(dvb + static_cast<int64_t>(r0) * p.ldv.row + c) = pack_bf16x2(dv[i][0], dv[i][1]);
    }
    if (r0 + 8 < p.Nk) {
      *reinterpret_cast<uint32_t*>(dkb + static_cast<int64_t>(r0 + 8) * p.ldk.row + c) =
          pack_bf16x2(dk[i][2] * p.scale, dk[i][3] * p.scale);
      *reinterpret_cast<uint32_t*>(dvb + static_cast<int64_t>(r0 + 8) * p.ldv.row + c) =
          pack_bf16x2(dv[i][2], dv[i][3]);
    }
  }
}


// ---------------------------------------------------------------- single-tile backward
// Nq <= 64 and Nk <= 64 (the feature attention: one (table row, head) per work item, all
// of its queries and keys in one tile). Persistent over items (blockIdx.x, + gridDim.x,
// ...), four CTAs per SM (<= 128 registers, ~41 KB of shared memory each) so that one
// CTA's loads overlap the others' tensor-core work. An item's Q, K, V, dO, O tiles and LSE
// are staged with cp.async; D_i = dO_i . O_i comes from the staged tiles (no separate
// pass over O and dO) and dS^T then reuses the O tile; dQ is written once in bf16. All
// layouts share one (i0, i1, i2) decomposition of the item index, done once per item in
// 32-bit arithmetic.
constexpr int kSmallTile = kBlkQ * 128;                          // one [64][64] bf16 tile
constexpr int kSmallSmem = 5 * kSmallTile + 2 * kBlkQ * 4;        // Q K V dO O(->dS^T), LSE, D
constexpr int kSmallCtasPerSm = 4;

__device__ __forceinline__ void cp_async4(void* smem, const void* gmem, int src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(src_bytes)
               : "memory");
}

__device__ __forceinline__ int64_t lay_off(const Layout3& l, int i0, int i1, int i2) {
  return static_cast<int64_t>(i0) * l.s0 + static_cast<int64_t>(i1) * l.s1 + static_cast<int64_t>(i2) * l.s2;
}

__global__ void __launch_bounds__(kAttnThreads, kSmallCtasPerSm) attn_bwd_small_kernel(AttnBwdParams p) {
  extern __shared__ __align__(1024) uint8_t dyn[];
  uint8_t* sq = dyn;
  uint8_t* sk = dyn + kSmallTile;
  uint8_t* sv = dyn + 2 * kSmallTile;
  uint8_t* sdo = dyn + 3 * kSmallTile;
  uint8_t* so = dyn + 4 * kSmallTile;  // O, then dS^T
  float* slse = reinterpret_cast<float*>(dyn + 5 * kSmallTile);
  float* sdv = slse + kBlkQ;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int d1 = p.lq.d1, d2 = p.lq.d2;
  for (int bh = blockIdx.x; bh < p.BH; bh += gridDim.x) {
    const int i2 = bh % d2, t = bh / d2, i1 = t % d1, i0 = t / d1;
    load_tile(sq, p.q + lay_off(p.lq, i0, i1, i2), p.lq.row, 0, p.Nq, p.q_d_valid, tid, kAttnThreads);
    load_tile(sk, p.k + lay_off(p.lk, i0, i1, i2), p.lk.row, 0, p.Nk, p.q_d_valid, tid, kAttnThreads);
    load_tile(sv, p.v + lay_off(p.lv, i0, i1, i2), p.lv.row, 0, p.Nk, p.q_d_valid, tid, kAttnThreads);
    load_tile(sdo, p.dout + lay_off(p.ldo, i0, i1, i2), p.ldo.row, 0, p.Nq, p.d_valid, tid, kAttnThreads);
    load_tile(so, p.o + lay_off(p.lo, i0, i1, i2), p.lo.row, 0, p.Nq, p.d_valid, tid, kAttnThreads);
    if (tid < kBlkQ) {
      const bool ok = tid < p.Nq;
      cp_async4(slse + tid, ok ? p.lse + static_cast<int64_t>(bh) * p.Nq + tid : p.lse, ok ? 4 : 0);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    {  // D_i = dO_i . O_i: two threads per row, 32 columns each (padding columns are zero)
      const int r = tid >> 1, half = tid & 1;
      float acc = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 a = *reinterpret_cast<const uint4*>(sdo + swz(r, half * 4 + c));
        const uint4 b = *reinterpret_cast<const uint4*>(so + swz(r, half * 4 + c));
        const uint32_t aa[4] = {a.x, a.y, a.z, a.w}, bb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) acc += bf16lo(aa[i]) * bf16lo(bb[i]) + bf16hi(aa[i]) * bf16hi(bb[i]);
      }
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      if (half == 0) sdv[r] = acc;
    }
    uint32_t kf[4][4], vf[4][4];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int r = warp * 16 + (lane & 15);
      const int c = kk * 2 + (lane >> 4);
      ldsm_x4(kf[kk], smem_u32(sk + swz(r, c)));
      ldsm_x4(vf[kk], smem_u32(sv + swz(r, c)));
    }
    __syncthreads();  // D complete, O tile free for dS^T
    float dk[8][4], dv[8][4], dqa[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;
    bwd_tile(sq, sdo, sk, so, slse, sdv, kf, vf, 0, 0, p.Nk, p.Nq, p.scale_log2, warp, lane, dk, dv, dqa);
    const int r0 = warp * 16 + (lane >> 2);
    __nv_bfloat16* dqh = p.dq16 + lay_off(p.ldq, i0, i1, i2);
    __nv_bfloat16* dkb = p.dk + lay_off(p.ldk, i0, i1, i2);
    __nv_bfloat16* dvb = p.dv + lay_off(p.ldv, i0, i1, i2);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = i * 8 + (lane & 3) * 2;
      if (c >= p.d_valid) continue;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = r0 + 8 * h;
        if (r < p.Nq)
          *reinterpret_cast<uint32_t*>(dqh + static_cast<int64_t>(r) * p.ldq.row + c) =
              pack_bf16x2(dqa[i][2 * h] * p.scale, dqa[i][2 * h + 1] * p.scale);
        if (r < p.Nk) {
          *reinterpret_cast<uint32_t*>(dkb + static_cast<int64_t>(r) * p.ldk.row + c) =
              pack_bf16x2(dk[i][2 * h] * p.scale, dk[i][2 * h + 1] * p.scale);
          *reinterpret_cast<uint32_t*>(dvb + static_cast<int64_t>(r) * p.ldv.row + c) =
              pack_bf16x2(dv[i][2 * h], dv[i][2 * h + 1]);
        }
      }
    }
    __syncthreads();  // all reads of this item's tiles done before the next item's loads
  }
}

// ---------------------------------------------------------------- host
static Layout3 to_layout(const std::vector<int64_t>& l) {
  TORCH_CHECK(l.size() == 6, "layout: [s0, s1, s2, row, d1, d2] expected");
  return Layout3{l[0], l[1], l[2], l[3], static_cast<int>(l[4]), static_cast<int>(l[5])};
}

static void check_bf16(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16, name, ": bf16 CUDA tensor expected");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name, ": 16-byte aligned base expected");
}

// q/k/v/o are base tensors (any shape); the layouts give element strides relative to their data_ptr.
void attn_fwd(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, torch::Tensor& o,
              const c10::optional<torch::Tensor>& lse, std::vector<int64_t> lq, std::vector<int64_t> lk,
              std::vector<int64_t> lv, std::vector<int64_t> lo, int64_t BH, int64_t Nq, int64_t Nk, int64_t d_valid,
              double scale) {
  check_bf16(q, "q");
  check_bf16(k, "k");
  check_bf16(v, "v");
  check_bf16(o, "o");
  TORCH_CHECK(d_valid > 0 && d_valid <= kD && d_valid % 8 == 0, "attn_fwd: head dim must be a multiple of 8, <= 64");
  const at::cuda::CUDAGuard guard(q.device());
  AttnFwdParams p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  p.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  p.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.lq = to_layout(lq);
  p.lk = to_layout(lk);
  p.lv = to_layout(lv);
  p.lo = to_layout(lo);
  TORCH_CHECK(p.lq.row % 8 == 0 && p.lk.row % 8 == 0 && p.lv.row % 8 == 0 && p.lq.s0 % 8 == 0 && p.lq.s1 % 8 == 0 &&
                  p.lq.s2 % 8 == 0 && p.lk.s0 % 8 == 0 && p.lk.s1 % 8 == 0 && p.lk.s2 % 8 == 0 &&
                  p.lv.s0 % 8 == 0 && p.lv.s1 % 8 == 0 && p.lv.s2 % 8 == 0,
              "attn_fwd: Q/K/V rows must start on 16-byte boundaries");
  p.BH = static_cast<int>(BH);
  p.Nq = static_cast<int>(Nq);
  p.Nk = static_cast<int>(Nk);
  p.d_valid = static_cast<int>(d_valid);
  p.q_d_valid = p.d_valid;
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  if (lse.has_value() && lse->defined()) {
    TORCH_CHECK(lse->scalar_type() == at::kFloat && lse->numel() >= BH * Nq, "attn_fwd: fp32 lse [BH, Nq]");
    p.lse = lse->data_ptr<float>();
  }
  if (BH == 0 || Nq == 0) return;
  TORCH_CHECK(Nk > 0, "attn_fwd: at least one key");
  TORCH_CHECK(BH < 65536 * 32768LL, "attn_fwd: too many heads");
  p.n_tiles_q = static_cast<int>((Nq + kBlkQ - 1) / kBlkQ);
  TORCH_CHECK(BH * p.n_tiles_q < 2147483647LL, "attention grid too large");
  dim3 grid(static_cast<unsigned>(BH * p.n_tiles_q));
  TORCH_CHECK(BH <= 2147483647LL, "attn_fwd: BH too large");
  if (Nk <= kBlkK)
    attn_fwd_kernel<1><<<grid, kAttnThreads, 0, at::cuda::getCurrentCUDAStream()>>>(p);
  else
    attn_fwd_kernel<2><<<grid, kAttnThreads, 0, at::cuda::getCurrentCUDAStream()>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// kv: int8 [.., 2E] rows (K columns first, V at +E); scales fp32 [.., 2H] (K heads, then V heads).
void attn_fwd_q8(const torch::Tensor& q, const torch::Tensor& kv, const torch::Tensor& scales, torch::Tensor& o,
                 const c10::optional<torch::Tensor>& lse, std::vector<int64_t> lq, std::vector<int64_t> lkv,
                 std::vector<int64_t> ls, std::vector<int64_t> lo, int64_t E, int64_t H, int64_t BH, int64_t Nq,
                 int64_t Nk, int64_t d_valid, double scale) {
  check_bf16(q, "q");
  check_bf16(o, "o");
  TORCH_CHECK(kv.is_cuda() && kv.scalar_type() == at::kChar, "attn_fwd_q8: int8 K/V");
  TORCH_CHECK(scales.is_cuda() && scales.scalar_type() == at::kFloat, "attn_fwd_q8: fp32 scales");
  TORCH_CHECK(d_valid > 0 && d_valid <= kD && d_valid % 8 == 0, "attn_fwd_q8: head dim multiple of 8, <= 64");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(kv.data_ptr()) % 8 == 0, "attn_fwd_q8: 8-byte aligned K/V");
  const at::cuda::CUDAGuard guard(q.device());
  if (BH == 0 || Nq == 0) return;
  TORCH_CHECK(Nk > 0, "attn_fwd_q8: at least one key");
  AttnQ8Params p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.k = kv.data_ptr<int8_t>();
  p.v = kv.data_ptr<int8_t>() + E;
  p.ks = scales.data_ptr<float>();
  p.vs = scales.data_ptr<float>() + H;
  p.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.lq = to_layout(lq);
  p.lkv = to_layout(lkv);
  p.ls = to_layout(ls);
  p.lo = to_layout(lo);
  TORCH_CHECK(p.lkv.row % 8 == 0 && p.lkv.s0 % 8 == 0 && p.lkv.s1 % 8 == 0 && p.lkv.s2 % 8 == 0,
              "attn_fwd_q8: K/V rows must be 8-byte aligned");
  p.BH = static_cast<int>(BH);
  p.Nq = static_cast<int>(Nq);
  p.Nk = static_cast<int>(Nk);
  p.d_valid = static_cast<int>(d_valid);
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  if (lse.has_value() && lse->defined()) {
    TORCH_CHECK(lse->scalar_type() == at::kFloat && lse->numel() >= BH * Nq, "attn_fwd_q8: fp32 lse [BH, Nq]");
    p.lse = lse->data_ptr<float>();
  }
  p.n_tiles_q = static_cast<int>((Nq + kBlkQ - 1) / kBlkQ);
  TORCH_CHECK(BH * p.n_tiles_q < 2147483647LL, "attention grid too large");
  dim3 grid(static_cast<unsigned>(BH * p.n_tiles_q));
  attn_fwd_q8_kernel<<<grid, kAttnThreads, 0, at::cuda::getCurrentCUDAStream()>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void attn_bwd(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, const torch::Tensor& o,
              const torch::Tensor& dout, const torch::Tensor& lse, torch::Tensor& dq, torch::Tensor& dk,
              torch::Tensor& dv, std::vector<int64_t> lq, std::vector<int64_t> lk, std::vector<int64_t> lv,
              std::vector<int64_t> lo, std::vector<int64_t> ldo, std::vector<int64_t> ldk, std::vector<int64_t> ldv,
              std::vector<int64_t> ldq, int64_t BH, int64_t Nq, int64_t Nk, int64_t d_valid, double scale,
              const c10::optional<torch::Tensor>& dq16) {
  for (auto* t : std::initializer_list<const torch::Tensor*>{&q, &k, &v, &o, &dout, &dk, &dv}) check_bf16(*t, "attn_bwd");
  const bool direct = dq16.has_value() && dq16->defined();
  if (direct) {
    check_bf16(*dq16, "attn_bwd dq16");
    TORCH_CHECK(Nk <= kBlkK, "attn_bwd: a bf16 dQ output needs the keys in one tile (Nk <= 64)");
    TORCH_CHECK(ldq[3] % 2 == 0 && ldq[0] % 2 == 0 && ldq[1] % 2 == 0 && ldq[2] % 2 == 0,
                "attn_bwd: bf16 dQ rows must be 4-byte aligned");
  } else {
    TORCH_CHECK(dq.is_cuda() && dq.scalar_type() == at::kFloat, "attn_bwd: dq must be a zeroed fp32 accumulator");
  }
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.numel() >= BH * Nq, "attn_bwd: fp32 lse");
  TORCH_CHECK(d_valid > 0 && d_valid <= kD && d_valid % 8 == 0, "attn_bwd: head dim must be a multiple of 8, <= 64");
  const at::cuda::CUDAGuard guard(q.device());
  if (BH == 0 || Nq == 0 || Nk == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (direct && Nq <= kBlkQ) {
    // single tile in both directions: the persistent kernel with staged tiles
    for (const auto* l : {&lq, &lk, &lv, &lo, &ldo})
      TORCH_CHECK((*l)[0] % 8 == 0 && (*l)[1] % 8 == 0 && (*l)[2] % 8 == 0 && (*l)[3] % 8 == 0,
                  "attn_bwd: Q / K / V / O / dO rows must be 16-byte aligned");
    for (const auto* l : {&lk, &lv, &lo, &ldo, &ldk, &ldv, &ldq})
      TORCH_CHECK((*l)[4] == lq[4] && (*l)[5] == lq[5], "attn_bwd: layouts must share the (d1, d2) item split");
    TORCH_CHECK(lq[4] > 0 && lq[5] > 0, "attn_bwd: layout d1, d2 must be positive");
    AttnBwdParams p{};
    p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
    p.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
    p.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
    p.o = reinterpret_cast<const __nv_bfloat16*>(o.data_ptr());
    p.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
    p.lse = lse.data_ptr<float>();
    p.dq16 = reinterpret_cast<__nv_bfloat16*>(dq16->data_ptr());
    p.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
    p.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
    p.lq = to_layout(lq);
    p.lk = to_layout(lk);
    p.lv = to_layout(lv);
    p.lo = to_layout(lo);
    p.ldo = to_layout(ldo);
    p.ldk = to_layout(ldk);
    p.ldv = to_layout(ldv);
    p.ldq = to_layout(ldq);
    p.BH = static_cast<int>(BH);
    p.Nq = static_cast<int>(Nq);
    p.Nk = static_cast<int>(Nk);
    p.d_valid = static_cast<int>(d_valid);
    p.q_d_valid = p.d_valid;
    p.scale = static_cast<float>(scale);
    p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
    p.n_tiles_k = 1;
    TORCH_CHECK(BH < 2147483647LL, "attention grid too large");
    const int dev = q.get_device();
    static int small_smem_set[64] = {0};  // once per device
    if (!small_smem_set[dev]) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          kSmallSmem));
      small_smem_set[dev] = 1;
    }
    const int sms = at::cuda::getDeviceProperties(dev)->multiProcessorCount;
    const int64_t grid = std::min<int64_t>(BH, static_cast<int64_t>(persistent_sms(sms)) * kSmallCtasPerSm);
    attn_bwd_small_kernel<<<static_cast<unsigned>(grid), kAttnThreads, kSmallSmem, stream>>>(p);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  auto dvec = torch::empty({BH * Nq}, lse.options());
  {
    const int64_t rows = BH * Nq;
    attn_bwd_dot_kernel<<<static_cast<unsigned>((rows + 255) / 256), 256, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
        to_layout(lo), to_layout(ldo), static_cast<int>(BH), static_cast<int>(Nq), static_cast<int>(d_valid),
        dvec.data_ptr<float>());
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  AttnBwdParams p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  p.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  p.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  p.lse = lse.data_ptr<float>();
  p.dvec = dvec.data_ptr<float>();
  p.dq = direct ? nullptr : dq.data_ptr<float>();
  p.dq16 = direct ? reinterpret_cast<__nv_bfloat16*>(dq16->data_ptr()) : nullptr;
  p.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  p.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  p.lq = to_layout(lq);
  p.lk = to_layout(lk);
  p.lv = to_layout(lv);
  p.ldo = to_layout(ldo);
  p.ldk = to_layout(ldk);
  p.ldv = to_layout(ldv);
  p.ldq = to_layout(ldq);
  p.BH = static_cast<int>(BH);
  p.Nq = static_cast<int>(Nq);
  p.Nk = static_cast<int>(Nk);
  p.d_valid = static_cast<int>(d_valid);
  p.q_d_valid = p.d_valid;
  p.scale = static_cast<float>(scale);
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  p.n_tiles_k = static_cast<int>((Nk + kBlkK - 1) / kBlkK);
  TORCH_CHECK(BH * p.n_tiles_k < 2147483647LL, "attention grid too large");
  dim3 grid(static_cast<unsigned>(BH * p.n_tiles_k));
  attn_bwd_kernel<<<grid, kAttnThreads, 0, stream>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace nori

namespace nori {
// ---------------------------------------------------------------- multi-shard int8 K/V forward
// Context-row-sharded inference: the keys of one table are split over up to 8 ranks and
// each rank's int8 K/V shard lives in its own (IPC-shared) memory. One query CTA walks the
// tiles of every shard in turn - peer shards are read over NVLink with plain loads and
// dequantised on the way into shared memory - so the online softmax (running max and sum)
// spans the whole context and the result needs no separate partial-softmax merge.
constexpr int kMaxShards = 8;
struct AttnShardsParams {
  const __nv_bfloat16* q;
  __nv_bfloat16* o;
  float* lse;
  const int8_t* kv[kMaxShards];     // shard base (K columns; V at +E)
  const float* sc[kMaxShards];      // shard scale base (K heads; V heads at +H)
  int nk[kMaxShards];               // keys per shard
  int64_t kv_s0[kMaxShards];        // per-shard table stride (elements)
  int64_t sc_s0[kMaxShards];
  Layout3 lq, lkv, ls, lo;          // lkv / ls: s1, s2, row strides shared by all shards
  int n_shards, E, H;
  int BH, Nq, d_valid, n_tiles_q;
  float scale_log2;
};

__global__ void __launch_bounds__(kAttnThreads) attn_fwd_q8_shards_kernel(AttnShardsParams p) {
  __shared__ __align__(128) uint8_t sq[kBlkQ * 128];
  __shared__ __align__(128) uint8_t sk[kBlkK * 128];
  __shared__ __align__(128) uint8_t sv[kBlkK * 128];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t bh = blockIdx.x / p.n_tiles_q;
  const int q0 = static_cast<int>(blockIdx.x % p.n_tiles_q) * kBlkQ;
  load_tile(sq, p.q + p.lq.offset(bh, 0), p.lq.row, q0, p.Nq, p.d_valid, tid, kAttnThreads);
  cp_async_commit();
  cp_async_wait<0>();
  // head decomposition for the per-shard offsets (table index i0 uses the shard's own stride)
  const int64_t i2 = bh % p.lkv.d2;
  const int64_t t = bh / p.lkv.d2;
  const int64_t i1 = t % p.lkv.d1;
  const int64_t i0 = t / p.lkv.d1;
  FwdState st;
  bool init = false;
  // flatten (shard, tile) into one sequence and prefetch one step ahead
  auto shard_base = [&](int sh, const int8_t*& kb, const float*& ksb) {
    kb = p.kv[sh] + i0 * p.kv_s0[sh] + i1 * p.lkv.s1 + i2 * p.lkv.s2;
    ksb = p.sc[sh] + i0 * p.sc_s0[sh] + i1 * p.ls.s1 + i2 * p.ls.s2;
  };
  int sh = 0, tt = 0;
  while (sh < p.n_shards && p.nk[sh] == 0) ++sh;
  Q8Stage nk_st, nv_st;
  if (sh < p.n_shards) {
    const int8_t* kb;
    const float* ksb;
    shard_base(sh, kb, ksb);
    q8_fetch(nk_st, kb, ksb, p.lkv.row, p.ls.row, 0, p.nk[sh], p.d_valid, tid);
    q8_fetch(nv_st, kb + p.E, ksb + p.H, p.lkv.row, p.ls.row, 0, p.nk[sh], p.d_valid, tid);
  }
  while (sh < p.n_shards) {
    const int cur_nk = p.nk[sh], cur_t = tt;
    q8_commit(nk_st, sk, tid);
    q8_commit(nv_st, sv, tid);
    // advance to the next (shard, tile) and start its loads before computing this one
    int nsh = sh, ntt = tt + 1;
    if (ntt * kBlkK >= cur_nk) {
      ntt = 0;
      ++nsh;
      while (nsh < p.n_shards && p.nk[nsh] == 0) ++nsh;
    }
    if (nsh < p.n_shards) {
      const int8_t* kb;
      const float* ksb;
      shard_base(nsh, kb, ksb);
      q8_fetch(nk_st, kb, ksb, p.lkv.row, p.ls.row, ntt * kBlkK, p.nk[nsh], p.d_valid, tid);
      q8_fetch(nv_st, kb + p.E, ksb + p.H, p.lkv.row, p.ls.row, ntt * kBlkK, p.nk[nsh], p.d_valid, tid);
    }
    __syncthreads();
    if (!init) {
      fwd_init(st, sq, warp, lane);
      init = true;
    }
    fwd_tile(st, sk, sv, cur_t * kBlkK, cur_nk, p.scale_log2, lane);
    __syncthreads();
    sh = nsh;
    tt = ntt;
  }
  if (init) fwd_store(st, p.o + p.lo.offset(bh, 0), p.lo.row, p.lse, bh, q0, p.Nq, p.d_valid, warp, lane);
}

void attn_fwd_q8_shards(const torch::Tensor& q, std::vector<int64_t> kv_ptrs, std::vector<int64_t> sc_ptrs,
                        std::vector<int64_t> nks, std::vector<int64_t> kv_s0, std::vector<int64_t> sc_s0,
                        torch::Tensor& o, const c10::optional<torch::Tensor>& lse, std::vector<int64_t> lq,
                        std::vector<int64_t> lkv, std::vector<int64_t> ls, std::vector<int64_t> lo, int64_t E,
                        int64_t H, int64_t BH, int64_t Nq, int64_t d_valid, double scale) {
  check_bf16(q, "q");
  check_bf16(o, "o");
  const size_t ns = kv_ptrs.size();
  TORCH_CHECK(ns >= 1 && ns <= static_cast<size_t>(kMaxShards) && sc_ptrs.size() == ns && nks.size() == ns &&
                  kv_s0.size() == ns && sc_s0.size() == ns,
              "attn_fwd_q8_shards: 1..8 shards with one pointer / size / stride each");
  TORCH_CHECK(d_valid > 0 && d_valid <= kD && d_valid % 8 == 0, "attn_fwd_q8_shards: head dim multiple of 8, <= 64");
  const at::cuda::CUDAGuard guard(q.device());
  if (BH == 0 || Nq == 0) return;
  AttnShardsParams p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.n_shards = static_cast<int>(ns);
  int64_t total = 0;
  for (size_t i = 0; i < ns; ++i) {
    TORCH_CHECK(kv_ptrs[i] % 8 == 0 && sc_ptrs[i] % 4 == 0, "attn_fwd_q8_shards: misaligned shard base");
    p.kv[i] = reinterpret_cast<const int8_t*>(kv_ptrs[i]);
    p.sc[i] = reinterpret_cast<const float*>(sc_ptrs[i]);
    p.nk[i] = static_cast<int>(nks[i]);
    p.kv_s0[i] = kv_s0[i];
    p.sc_s0[i] = sc_s0[i];
    total += nks[i];
  }
  TORCH_CHECK(total > 0, "attn_fwd_q8_shards: at least one key");
  p.lq = to_layout(lq);
  p.lkv = to_layout(lkv);
  p.ls = to_layout(ls);
  p.lo = to_layout(lo);
  TORCH_CHECK(p.lkv.row % 8 == 0 && p.lkv.s1 % 8 == 0 && p.lkv.s2 % 8 == 0, "attn_fwd_q8_shards: 8-byte K/V rows");
  p.E = static_cast<int>(E);
  p.H = static_cast<int>(H);
  p.BH = static_cast<int>(BH);
  p.Nq = static_cast<int>(Nq);
  p.d_valid = static_cast<int>(d_valid);
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  if (lse.has_value() && lse->defined()) p.lse = lse->data_ptr<float>();
  p.n_tiles_q = static_cast<int>((Nq + kBlkQ - 1) / kBlkQ);
  attn_fwd_q8_shards_kernel<<<static_cast<unsigned>(BH * p.n_tiles_q), kAttnThreads, 0,
                              at::cuda::getCurrentCUDAStream()>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Plain-load copy of a row-strided 2-D region (e.g. a peer's K/V columns) into local memory.
__global__ void copy_rows_kernel(const uint8_t* __restrict__ src, int64_t src_ld, uint8_t* __restrict__ dst,
                                 int64_t dst_ld, int64_t rows, int64_t row_bytes) {
  const int64_t chunks = row_bytes / 16;
  const int64_t total = rows * chunks;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / chunks, c = i % chunks;
    *reinterpret_cast<uint4*>(dst + r * dst_ld + c * 16) = *reinterpret_cast<const uint4*>(src + r * src_ld + c * 16);
  }
}

void copy_rows(int64_t src_ptr, int64_t src_ld_bytes, torch::Tensor& dst, int64_t dst_ld_bytes, int64_t rows,
               int64_t row_bytes) {
  TORCH_CHECK(dst.is_cuda(), "copy_rows: CUDA destination");
  TORCH_CHECK(src_ptr % 16 == 0 && reinterpret_cast<uintptr_t>(dst.data_ptr()) % 16 == 0 && src_ld_bytes % 16 == 0 &&
                  dst_ld_bytes % 16 == 0 && row_bytes % 16 == 0,
              "copy_rows: 16-byte aligned rows");
  const at::cuda::CUDAGuard guard(dst.device());
  if (rows == 0 || row_bytes == 0) return;
  const int64_t total = rows * (row_bytes / 16);
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 148 * 8));
  copy_rows_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint8_t*>(src_ptr), src_ld_bytes, reinterpret_cast<uint8_t*>(dst.data_ptr()),
      dst_ld_bytes, rows, row_bytes);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Dvec = rowsum(dO * O) for the tensor-core backward (same kernel as attn_bwd's first step).
torch::Tensor attn_dvec(const torch::Tensor& o, const torch::Tensor& dout, std::vector<int64_t> lo,
                        std::vector<int64_t> ldo, int64_t BH, int64_t Nq, int64_t d_valid) {
  check_bf16(o, "o");
  check_bf16(dout, "dout");
  TORCH_CHECK(d_valid > 0 && d_valid <= kD && d_valid % 8 == 0, "attn_dvec: head dim multiple of 8, <= 64");
  const at::cuda::CUDAGuard guard(o.device());
  auto dvec = torch::empty({BH * Nq}, o.options().dtype(at::kFloat));
  if (BH * Nq == 0) return dvec;
  const int64_t rows = BH * Nq;
  attn_bwd_dot_kernel<<<static_cast<unsigned>((rows + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
      to_layout(lo), to_layout(ldo), static_cast<int>(BH), static_cast<int>(Nq), static_cast<int>(d_valid),
      dvec.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dvec;
}
}  // namespace nori

// ---------------------------------------------------------------- allocation-free variant
// See nori_noalloc.h. The scratch for the dO . O row products lives in this file-scope
// device array; host code must not pass `g_noalloc_dvec` itself to a kernel (on the host
// it names a host-side shadow), only the address returned by cudaGetSymbolAddress.
#include <mutex>
#include <string>

#include "nori_noalloc.h"

namespace {
static __device__ __align__(256) float g_noalloc_dvec[NORI_NOALLOC_MAX_ROWS];

constexpr int kMaxDevices = 64;
float* g_noalloc_addr[kMaxDevices] = {nullptr};
std::mutex g_noalloc_mutex;
thread_local std::string g_noalloc_error;

cudaError_t noalloc_fail(const char* why) {
  g_noalloc_error = why;
  return cudaErrorInvalidValue;
}

nori::Layout3 layout_from(const int64_t* l) {
  return nori::Layout3{l[0], l[1], l[2], l[3], static_cast<int>(l[4]), static_cast<int>(l[5])};
}
}  // namespace

extern "C" __attribute__((visibility("default"))) const char* nori_attention_bwd_noalloc_error(void) {
  return g_noalloc_error.c_str();
}

extern "C" __attribute__((visibility("default"))) cudaError_t nori_attention_bwd_noalloc(
    const void* q, const void* k, const void* v, const void* o, const void* dout, const float* lse, float* dq, void* dk,
    void* dv, const int64_t* lq, const int64_t* lk, const int64_t* lv, const int64_t* lo, const int64_t* ldo,
    const int64_t* ldk, const int64_t* ldv, int64_t BH, int64_t Nq, int64_t Nk, int64_t d_valid, double scale,
    cudaStream_t stream) {
  g_noalloc_error.clear();
  // Every check runs before anything is queued: a rejected call changes nothing.
  if (!q || !k || !v || !o || !dout || !lse || !dq || !dk || !dv || !lq || !lk || !lv || !lo || !ldo || !ldk || !ldv)
    return noalloc_fail("nori_attention_bwd_noalloc: null pointer argument");
  if (BH < 0 || Nq < 0 || Nk < 0) return noalloc_fail("nori_attention_bwd_noalloc: negative size");
  const int64_t kMax = static_cast<int64_t>(NORI_NOALLOC_MAX_ROWS);
  if (BH > kMax || Nq > kMax || BH * Nq > kMax)  // each factor bounded first: the product cannot overflow
    return noalloc_fail("nori_attention_bwd_noalloc: BH * Nq exceeds NORI_NOALLOC_MAX_ROWS (1048576)");
  if (Nk > 2147483647LL) return noalloc_fail("nori_attention_bwd_noalloc: Nk too large");
  if (d_valid <= 0 || d_valid > nori::kD || d_valid % 8 != 0)
    return noalloc_fail("nori_attention_bwd_noalloc: head dim must be a multiple of 8, at most 64");
  // the kernels move bf16 rows in 16-byte vectors and dq in float4s
  for (const void* ptr : {q, k, v, o, dout, static_cast<const void*>(dq), static_cast<const void*>(dk),
                          static_cast<const void*>(dv)})
    if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0)
      return noalloc_fail("nori_attention_bwd_noalloc: q, k, v, o, dout, dq, dk and dv must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(lse) % 4 != 0)
    return noalloc_fail("nori_attention_bwd_noalloc: lse must be 4-byte aligned");
  for (const int64_t* l : {lq, lk, lv, lo, ldo, ldk, ldv}) {
    if (l[0] < 0 || l[1] < 0 || l[2] < 0 || l[3] < 0 || l[0] % 8 || l[1] % 8 || l[2] % 8 || l[3] % 8)
      return noalloc_fail("nori_attention_bwd_noalloc: layout strides must be non-negative multiples of 8 elements");
    if (l[4] <= 0 || l[5] <= 0 || l[4] > 2147483647LL || l[5] > 2147483647LL)
      return noalloc_fail("nori_attention_bwd_noalloc: layout d1 and d2 must be positive and fit in 32 bits");
  }
  if (BH == 0 || Nq == 0 || Nk == 0) return cudaSuccess;
  const int64_t n_tiles_k = (Nk + nori::kBlkK - 1) / nori::kBlkK;
  if (BH * n_tiles_k >= 2147483647LL) return noalloc_fail("nori_attention_bwd_noalloc: grid too large");
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= kMaxDevices) return noalloc_fail("nori_attention_bwd_noalloc: device index out of range");
  float* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_addr[dev] == nullptr) {
      // once per device, with that device current
      err = cudaGetSymbolAddress(reinterpret_cast<void**>(&g_noalloc_addr[dev]), g_noalloc_dvec);
      if (err != cudaSuccess) {
        g_noalloc_addr[dev] = nullptr;
        return err;
      }
    }
    scratch = g_noalloc_addr[dev];
  }
  // the query-gradient accumulator must start at zero
  err = cudaMemsetAsync(dq, 0, static_cast<size_t>(BH * Nq * nori::kD) * sizeof(float), stream);
  if (err != cudaSuccess) return err;
  const int64_t rows = BH * Nq;
  nori::attn_bwd_dot_kernel<<<static_cast<unsigned>((rows + 255) / 256), 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(o), reinterpret_cast<const __nv_bfloat16*>(dout), layout_from(lo),
      layout_from(ldo), static_cast<int>(BH), static_cast<int>(Nq), static_cast<int>(d_valid), scratch);
  err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  nori::AttnBwdParams p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(q);
  p.k = reinterpret_cast<const __nv_bfloat16*>(k);
  p.v = reinterpret_cast<const __nv_bfloat16*>(v);
  p.dout = reinterpret_cast<const __nv_bfloat16*>(dout);
  p.lse = lse;
  p.dvec = scratch;
  p.dq = dq;
  p.dk = reinterpret_cast<__nv_bfloat16*>(dk);
  p.dv = reinterpret_cast<__nv_bfloat16*>(dv);
  p.lq = layout_from(lq);
  p.lk = layout_from(lk);
  p.lv = layout_from(lv);
  p.ldo = layout_from(ldo);
  p.ldk = layout_from(ldk);
  p.ldv = layout_from(ldv);
  p.ldq = nori::Layout3{Nq * nori::kD, 0, 0, nori::kD, 1, 1};
  p.BH = static_cast<int>(BH);
  p.Nq = static_cast<int>(Nq);
  p.Nk = static_cast<int>(Nk);
  p.d_valid = static_cast<int>(d_valid);
  p.q_d_valid = p.d_valid;
  p.scale = static_cast<float>(scale);
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  p.n_tiles_k = static_cast<int>(n_tiles_k);
  nori::attn_bwd_kernel<<<static_cast<unsigned>(BH * p.n_tiles_k), nori::kAttnThreads, 0, stream>>>(p);
  return cudaGetLastError();
}
