// Query-aware scalable softmax (QASS) rescale of the sequence-attention queries,
// forward and backward, fused per 16 query vectors per warp.
//
//   q' = q * s[h] * (1 + tanh(W2 gelu(W1 q + b1) + b2))        (reference
//   model/layer.py:316-456, mode "full"; "base_only" drops the gate factor)
//
// q is one head's D-vector of a token-major row (D <= 64, zero padded to 64); the gate
// MLP (D -> 64 -> D, exact-erf GELU) runs on mma.m16n8k16 with both weight matrices in
// shared memory; s [H, D] is the per-head base scale log n (1 + tanh(base(log n)))
// computed once per call on the host side.
//
// The backward kernel recomputes the gate, writes dq (bf16, into the caller's strided
// gradient buffer) and reduces ds [H, D], db1, db2, dW1, dW2 across all vectors:
// every 128 vectors the CTA stages (dz2, gelu) and (dz1, q) in shared memory and four
// warps each accumulate a 16-row slice of dW2 and dW1 on the tensor cores.
//
// With the gate MLP and 128 % H == 0, H <= 16, both entry points run the tcgen05 kernels
// of qass_tc.cu instead (environment NORI_QASS_TC=0 selects these for comparison); the
// kernels below serve the other head counts and the gate-free modes.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "sm100.cuh"

namespace nori {
namespace qass {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kVec = 16;                       // vectors per warp step
constexpr int kStageVec = kWarps * kVec;       // 128 vectors per CTA step

__device__ __forceinline__ int swz(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

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

__device__ __forceinline__ float gelu(float z) { return 0.5f * z * (1.0f + erff(z * 0.70710678118654752f)); }
// tanh(x) = 1 - 2 / (1 + e^(2x)) with the fast exponential and division intrinsics: absolute
// error ~1e-7 (the gate only uses 1 + tanh and 1 - tanh^2, where that is far below bf16
// resolution); saturates to +-1 for large |x|.
__device__ __forceinline__ float tanh_fast(float x) { return 1.0f - __fdividef(2.0f, 1.0f + __expf(2.0f * x)); }

// gelu(z) and gelu'(z) from one erf evaluation (the backward needs both)
__device__ __forceinline__ void gelu_and_grad(float z, float& g, float& dg) {
  const float cdf = 0.5f * (1.0f + erff(z * 0.70710678118654752f));
  g = z * cdf;
  dg = cdf + z * 0.3989422804014327f * __expf(-0.5f * z * z);
}

// A fragments of a [16 x 64] bf16 tile (rows = vectors) stored swizzled at `tile`.
__device__ __forceinline__ void load_a(uint32_t (&a)[4][4], const uint8_t* tile, int lane) {
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) ldsm_x4(a[kk], smem_u32(tile + swz(lane & 15, kk * 2 + (lane >> 4))));
}

// acc[16 x 64] += A[16 x 64] * B, B[k][n] = M[n][k] for a row-major [64 n][64 k] matrix M (non-trans loads)
__device__ __forceinline__ void mma_nt(float (&acc)[8][4], const uint32_t (&a)[4][4], const uint8_t* M, int lane) {
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
    for (int j2 = 0; j2 < 4; ++j2) {
      uint32_t b[4];
      const int n = j2 * 16 + (lane & 7) + ((lane >> 4) << 3);
      const int c = kk * 2 + ((lane >> 3) & 1);
      ldsm_x4(b, smem_u32(M + swz(n, c)));
      mma16816(acc[2 * j2], a[kk], b[0], b[1]);
      mma16816(acc[2 * j2 + 1], a[kk], b[2], b[3]);
    }
  }
}

// acc[16 x 64] += A[16 x 64] * B, B[k][n] = M[k][n] for a row-major [64 k][64 n] matrix M (trans loads)
__device__ __forceinline__ void mma_nn(float (&acc)[8][4], const uint32_t (&a)[4][4], const uint8_t* M, int lane) {
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
    for (int i2 = 0; i2 < 4; ++i2) {
      uint32_t b[4];
      const int k = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
      const int c = i2 * 2 + (lane >> 4);
      ldsm_x4_t(b, smem_u32(M + swz(k, c)));
      mma16816(acc[2 * i2], a[kk], b[0], b[1]);
      mma16816(acc[2 * i2 + 1], a[kk], b[2], b[3]);
    }
  }
}

// accumulator [16 x 64] (C layout) -> A fragments (bf16)
__device__ __forceinline__ void acc_to_a(const float (&c)[8][4], uint32_t (&a)[4][4]) {
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    a[kk][0] = pack_bf16x2(c[2 * kk][0], c[2 * kk][1]);
    a[kk][1] = pack_bf16x2(c[2 * kk][2], c[2 * kk][3]);
    a[kk][2] = pack_bf16x2(c[2 * kk + 1][0], c[2 * kk + 1][1]);
    a[kk][3] = pack_bf16x2(c[2 * kk + 1][2], c[2 * kk + 1][3]);
  }
}

// accumulator [16 x 64] -> bf16 swizzled smem tile
__device__ __forceinline__ void acc_to_smem(const float (&c)[8][4], uint8_t* tile, int lane) {
  const int g = lane >> 2, cc = (lane & 3) * 2;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int col = i * 8 + cc;
    *reinterpret_cast<uint32_t*>(tile + swz(g, col >> 3) + (col & 7) * 2) = pack_bf16x2(c[i][0], c[i][1]);
    *reinterpret_cast<uint32_t*>(tile + swz(g + 8, col >> 3) + (col & 7) * 2) = pack_bf16x2(c[i][2], c[i][3]);
  }
}

struct Params {
  const __nv_bfloat16* q;  // [R, ldq], head h at column h * D
  int64_t ldq;
  __nv_bfloat16* out;  // forward: [R, ldo]; backward: dq (bf16) [R, ldo]
  int64_t ldo;
  const float* dout;  // backward: dq' fp32 [R, ldd]
  int64_t ldd;
  const float* s;     // [H, D]
  const float* w1;    // [64, D]
  const float* b1;    // [64]
  const float* w2;    // [D, 64]
  const float* b2;    // [D]
  float* gs;          // backward: ds [H, D]
  float* gw1;         // [64, D]
  float* gb1;         // [64]
  float* gw2;         // [D, 64]
  float* gb2;         // [D]
  int64_t R;
  int H, D, gate;
};

// vector index -> (token row, head) in 32-bit arithmetic (a 64-bit division is a long
// software sequence on the GPU); the host checks R * H < 2^31
__device__ __forceinline__ void vec_split(int64_t v, int H, int64_t& row, int& h) {
  const unsigned vv = static_cast<unsigned>(v), hh = static_cast<unsigned>(H);
  const unsigned rr = vv / hh;
  row = rr;
  h = static_cast<int>(vv - rr * hh);
}

// stage weights as bf16 swizzled [64][64]: W1 rows = hidden j (cols d), W2 rows = d (cols j)
__device__ __forceinline__ void stage_weights(const Params& p, uint8_t* sW1, uint8_t* sW2, float* sb1, float* sb2,
                                              float* ss) {
  for (int i = threadIdx.x; i < 64 * 64; i += blockDim.x) {
    const int r = i >> 6, c = i & 63;
    const float w1 = (c < p.D) ? p.w1[r * p.D + c] : 0.f;
    const float w2 = (r < p.D) ? p.w2[r * 64 + c] : 0.f;
    reinterpret_cast<__nv_bfloat16*>(sW1 + swz(r, c >> 3))[c & 7] = __float2bfloat16(w1);
    reinterpret_cast<__nv_bfloat16*>(sW2 + swz(r, c >> 3))[c & 7] = __float2bfloat16(w2);
  }
  for (int i = threadIdx.x; i < 64; i += blockDim.x) {
    sb1[i] = p.b1 ? p.b1[i] : 0.f;
    sb2[i] = (p.b2 && i < p.D) ? p.b2[i] : 0.f;
  }
  for (int i = threadIdx.x; i < p.H * 64; i += blockDim.x) {
    const int h = i >> 6, d = i & 63;
    ss[i] = d < p.D ? p.s[h * p.D + d] : 0.f;
  }
}

// 16 vectors (v0 .. v0+15) of q into a swizzled [16][64] tile (zero padded)
__device__ __forceinline__ void load_q(const Params& p, int64_t v0, uint8_t* tile, int lane) {
  for (int i = lane; i < 16 * 8; i += 32) {
    const int r = i >> 3, c = i & 7;
    const int64_t v = v0 + r;
    uint4 w = make_uint4(0u, 0u, 0u, 0u);
    if (v < p.R * p.H && c * 8 < p.D) {
      int64_t row;
      int h;
      vec_split(v, p.H, row, h);
      w = *reinterpret_cast<const uint4*>(p.q + row * p.ldq + h * p.D + c * 8);
    }
    *reinterpret_cast<uint4*>(tile + swz(r, c)) = w;
  }
  __syncwarp();
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// Asynchronous copy of the 16-vector q tile starting at v0 into a swizzled [16][64] tile;
// vectors past the end are zero-filled, the head-dim padding chunks (>= D/8) are never
// written (zeroed once by the caller).
__device__ __forceinline__ void prefetch_q(const Params& p, int64_t v0, uint8_t* tile, int lane) {
  const int nc = p.D >> 3;
  const int64_t nvec = p.R * p.H;
  for (int i = lane; i < 16 * 8; i += 32) {
    const int r = i >> 3, c = i & 7;
    if (c >= nc) continue;
    const int64_t v = v0 + r;
    const bool ok = v < nvec;
    int64_t row = 0;
    int h = 0;
    if (ok) vec_split(v, p.H, row, h);
    const __nv_bfloat16* src = ok ? p.q + row * p.ldq + h * p.D + c * 8 : p.q;
    cp_async16(tile + swz(r, c), src, ok ? 16 : 0);
  }
}

// Zero the head-dim padding chunks (columns >= D) of a swizzled [16][64] tile.
__device__ __forceinline__ void zero_q_pad(const Params& p, uint8_t* tile, int lane) {
  for (int i = lane; i < 16 * 8; i += 32) {
    const int r = i >> 3, c = i & 7;
    if (c >= (p.D >> 3)) *reinterpret_cast<uint4*>(tile + swz(r, c)) = make_uint4(0u, 0u, 0u, 0u);
  }
}

constexpr int kDoutLd = 68;  // fp32 row stride of a dout tile (padding spreads the banks)

// Asynchronous copy of the 16 fp32 gradient vectors starting at v0 into a [16][kDoutLd] tile.
__device__ __forceinline__ void prefetch_dout(const Params& p, int64_t v0, float* tile, int lane) {
  const int nc = p.D >> 2;
  const int64_t nvec = p.R * p.H;
  for (int i = lane; i < 16 * 16; i += 32) {
    const int r = i >> 4, c = i & 15;
    if (c >= nc) continue;
    const int64_t v = v0 + r;
    const bool ok = v < nvec;
    int64_t row = 0;
    int h = 0;
    if (ok) vec_split(v, p.H, row, h);
    const float* src = ok ? p.dout + row * p.ldd + h * p.D + c * 4 : p.dout;
    cp_async16(tile + r * kDoutLd + c * 4, src, ok ? 16 : 0);
  }
}

__global__ void __launch_bounds__(kThreads) qass_fwd_kernel(Params p) {
  __shared__ __align__(128) uint8_t sW1[64 * 128];
  __shared__ __align__(128) uint8_t sW2[64 * 128];
  __shared__ float sb1[64], sb2[64];
  // dynamic: double-buffered q tiles per warp [kWarps][2][16 x 64] bf16, then ss [H][64]
  extern __shared__ __align__(128) uint8_t dynf[];
  uint8_t (*sQ2)[2][16 * 128] = reinterpret_cast<uint8_t (*)[2][16 * 128]>(dynf);
  float* ss = reinterpret_cast<float*>(dynf + kWarps * 2 * 16 * 128);
  stage_weights(p, sW1, sW2, sb1, sb2, ss);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, cc = (lane & 3) * 2;
  const int64_t nvec = p.R * p.H;
  const int64_t vstep = static_cast<int64_t>(gridDim.x) * kWarps * kVec;
  int buf = 0;
  zero_q_pad(p, sQ2[warp][0], lane);
  zero_q_pad(p, sQ2[warp][1], lane);
  prefetch_q(p, (static_cast<int64_t>(blockIdx.x) * kWarps + warp) * kVec, sQ2[warp][0], lane);
  cp_async_commit();
  for (int64_t v0 = (static_cast<int64_t>(blockIdx.x) * kWarps + warp) * kVec; v0 < nvec; v0 += vstep, buf ^= 1) {
    // the next group's tile loads while this one is computed
    if (v0 + vstep < nvec) prefetch_q(p, v0 + vstep, sQ2[warp][buf ^ 1], lane);
    cp_async_commit();
    cp_async_wait1();
    __syncwarp();
    uint8_t* const sQw = sQ2[warp][buf];
    float t[8][4];
    if (p.gate) {
      uint32_t a[4][4];
      load_a(a, sQw, lane);
      float z1[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) z1[i][e] = sb1[i * 8 + cc + (e & 1)];
      mma_nt(z1, a, sW1, lane);
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) z1[i][e] = gelu(z1[i][e]);
      acc_to_a(z1, a);
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) t[i][e] = sb2[i * 8 + cc + (e & 1)];
      mma_nt(t, a, sW2, lane);
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) t[i][e] = 1.0f + tanh_fast(t[i][e]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) t[i][0] = t[i][1] = t[i][2] = t[i][3] = 1.0f;
    }
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int64_t v = v0 + g + half * 8;
      if (v >= nvec) continue;
      int64_t row;
      int h;
      vec_split(v, p.H, row, h);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int d = i * 8 + cc;
        if (d >= p.D) continue;
        const uint8_t* base = sQw + swz(g + half * 8, d >> 3) + (d & 7) * 2;
        const uint32_t qq = *reinterpret_cast<const uint32_t*>(base);
        const float o0 = bf16lo(qq) * ss[h * 64 + d] * t[i][half * 2];
        const float o1 = bf16hi(qq) * ss[h * 64 + d + 1] * t[i][half * 2 + 1];
        *reinterpret_cast<uint32_t*>(p.out + row * p.ldo + h * p.D + d) = pack_bf16x2(o0, o1);
      }
    }
    __syncwarp();
  }
}

__global__ void __launch_bounds__(kThreads) qass_bwd_kernel(Params p) {
  __shared__ __align__(128) uint8_t sW1[64 * 128];
  __shared__ __align__(128) uint8_t sW2[64 * 128];
  __shared__ float sb1[64], sb2[64], gb1[64], gb2[64];
  // dynamic: staging for the weight-gradient products ([128 vectors][64] bf16 each,
  // swizzled), then ss [H][64] and gs [H][64]
  extern __shared__ __align__(128) uint8_t dyn[];
  uint8_t* sDz2 = dyn;
  uint8_t* sAct = sDz2 + kStageVec * 128;
  uint8_t* sDz1 = sAct + kStageVec * 128;
  uint8_t* sQs = sDz1 + kStageVec * 128;
  uint8_t* sQ2 = sQs + kStageVec * 128;                               // [kWarps][2][16 x 64] bf16 q tiles
  float* sDo2 = reinterpret_cast<float*>(sQ2 + kWarps * 2 * 16 * 128);  // [kWarps][2][16 x kDoutLd] fp32
  float* ss = sDo2 + kWarps * 2 * 16 * kDoutLd;
  float* gsm = ss + p.H * 64;
  stage_weights(p, sW1, sW2, sb1, sb2, ss);
  for (int i = threadIdx.x; i < 64; i += blockDim.x) gb1[i] = gb2[i] = 0.f;
  for (int i = threadIdx.x; i < p.H * 64; i += blockDim.x) gsm[i] = 0.f;
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, cc = (lane & 3) * 2;
  const int64_t nvec = p.R * p.H;
  // per-warp weight-gradient slices: warps 0-3 own dW2 rows [16w, 16w+16) (d), warps 4-7 own dW1 rows (j)
  float wacc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) wacc[i][0] = wacc[i][1] = wacc[i][2] = wacc[i][3] = 0.f;
  // ds partial sums: when H divides 8 every vector this thread touches has head (g % H),
  // so the per-(h, d) sums stay in registers (16 columns per thread)
  const bool ds_in_regs = (8 % p.H) == 0;
  float dsacc[8][2];
#pragma unroll
  for (int i = 0; i < 8; ++i) dsacc[i][0] = dsacc[i][1] = 0.f;
  const int64_t step = static_cast<int64_t>(gridDim.x) * kStageVec;
  uint8_t* const sQa = sQ2 + warp * 2 * 16 * 128;
  float* const sDoa = sDo2 + warp * 2 * 16 * kDoutLd;
  int buf = 0;
  zero_q_pad(p, sQa, lane);
  zero_q_pad(p, sQa + 16 * 128, lane);
  {
    const int64_t v_first = static_cast<int64_t>(blockIdx.x) * kStageVec + warp * kVec;
    prefetch_q(p, v_first, sQa, lane);
    prefetch_dout(p, v_first, sDoa, lane);
    cp_async_commit();
  }
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * kStageVec; base < nvec; base += step, buf ^= 1) {
    const int64_t v0 = base + warp * kVec;
    // the next step's q and gradient tiles load while this step is computed
    if (base + step < nvec) {
      prefetch_q(p, v0 + step, sQa + (buf ^ 1) * 16 * 128, lane);
      prefetch_dout(p, v0 + step, sDoa + (buf ^ 1) * 16 * kDoutLd, lane);
    }
    cp_async_commit();
    cp_async_wait1();
    __syncwarp();
    uint8_t* const sQw = sQa + buf * 16 * 128;
    const float* const sDow = sDoa + buf * 16 * kDoutLd;
    uint32_t aq[4][4];
    load_a(aq, sQw, lane);
    float z1[8][4], z2[8][4];
    float act[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        z1[i][e] = sb1[i * 8 + cc + (e & 1)];
        z2[i][e] = sb2[i * 8 + cc + (e & 1)];
      }
    if (p.gate) {
      mma_nt(z1, aq, sW1, lane);
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float g, dg;
          gelu_and_grad(z1[i][e], g, dg);
          act[i][e] = g;
          z1[i][e] = dg;  // z1 is only needed through gelu'(z1) from here on
        }
      uint32_t aa[4][4];
      acc_to_a(act, aa);
      mma_nt(z2, aa, sW2, lane);
    }
    // dq' -> du, dz2, direct dq, ds
    float dz2[8][4], dqd[8][4];
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int64_t v = v0 + g + half * 8;
      const bool ok = v < nvec;
      int64_t row_unused = 0;
      int h = 0;
      if (ok) vec_split(v, p.H, row_unused, h);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
#pragma unroll
        for (int e2 = 0; e2 < 2; ++e2) {
          const int d = i * 8 + cc + e2;
          const int e = half * 2 + e2;
          float dqp = 0.f, x = 0.f;
          if (ok && d < p.D) {
            dqp = sDow[(g + half * 8) * kDoutLd + d];
            const __nv_bfloat16* qt =
                reinterpret_cast<const __nv_bfloat16*>(sQw + swz(g + half * 8, d >> 3) + (d & 7) * 2);
            x = __bfloat162float(*qt);
          }
          const float sv = ss[h * 64 + (d < 64 ? d : 0)];
          const float t = p.gate ? tanh_fast(z2[i][e]) : 0.f;
          const float gate = 1.0f + t;
          dqd[i][e] = dqp * gate * sv;
          if (ok && d < p.D) {
            if (ds_in_regs)
              dsacc[i][e2] += dqp * gate * x;
            else
              atomicAdd(&gsm[h * 64 + d], dqp * gate * x);
          }
          dz2[i][e] = p.gate ? dqp * x * sv * (1.0f - t * t) : 0.f;
        }
      }
    }
    float dq[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) dq[i][e] = dqd[i][e];
    if (p.gate) {
      // db2
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float s0 = dz2[i][0] + dz2[i][2], s1 = dz2[i][1] + dz2[i][3];
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          s0 += __shfl_xor_sync(0xffffffffu, s0, o);
          s1 += __shfl_xor_sync(0xffffffffu, s1, o);
        }
        if (g == 0) {
          atomicAdd(&gb2[i * 8 + cc], s0);
          atomicAdd(&gb2[i * 8 + cc + 1], s1);
        }
      }
      // dh = dz2 W2 ([16 x d] x [d x j]) : B[k=d][n=j] = W2[d][j] -> trans loads of W2 rows
      uint32_t adz2[4][4];
      acc_to_a(dz2, adz2);
      float dh[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) dh[i][0] = dh[i][1] = dh[i][2] = dh[i][3] = 0.f;
      mma_nn(dh, adz2, sW2, lane);
      float dz1[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) dz1[i][e] = dh[i][e] * z1[i][e];  // z1 holds gelu'(z1)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float s0 = dz1[i][0] + dz1[i][2], s1 = dz1[i][1] + dz1[i][3];
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          s0 += __shfl_xor_sync(0xffffffffu, s0, o);
          s1 += __shfl_xor_sync(0xffffffffu, s1, o);
        }
        if (g == 0) {
          atomicAdd(&gb1[i * 8 + cc], s0);
          atomicAdd(&gb1[i * 8 + cc + 1], s1);
        }
      }
      // dq += dz1 W1 ([16 x j] x [j x d]) : B[k=j][n=d] = W1[j][d] -> trans loads of W1 rows
      uint32_t adz1[4][4];
      acc_to_a(dz1, adz1);
      mma_nn(dq, adz1, sW1, lane);
      // stage for the weight-gradient products (rows = vectors of this CTA step)
      acc_to_smem(dz2, sDz2 + warp * 16 * 128, lane);
      acc_to_smem(act, sAct + warp * 16 * 128, lane);
      acc_to_smem(dz1, sDz1 + warp * 16 * 128, lane);
      for (int i = lane; i < 16 * 8; i += 32) {  // copy the q tile (already swizzled by row within 16)
        const int r = i >> 3, c = i & 7;
        *reinterpret_cast<uint4*>(sQs + swz(warp * 16 + r, c)) = *reinterpret_cast<const uint4*>(sQw + swz(r, c));
      }
    }
    // write dq (bf16)
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int64_t v = v0 + g + half * 8;
      if (v >= nvec) continue;
      int64_t row;
      int h;
      vec_split(v, p.H, row, h);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int d = i * 8 + cc;
        if (d >= p.D) continue;
        *reinterpret_cast<uint32_t*>(p.out + row * p.ldo + h * p.D + d) =
            pack_bf16x2(dq[i][half * 2], dq[i][half * 2 + 1]);
      }
    }
    if (p.gate) {
      __syncthreads();
      // dW2[d][j] += sum_v dz2[v][d] act[v][j]  (warps 0-3: d rows 16w..)
      // dW1[j][d] += sum_v dz1[v][j] q[v][d]    (warps 4-7: j rows 16(w-4)..)
      const uint8_t* Lhs = warp < 4 ? sDz2 : sDz1;
      const uint8_t* Rhs = warp < 4 ? sAct : sQs;
      const int m0 = (warp & 3) * 16;
#pragma unroll
      for (int kk = 0; kk < kStageVec / 16; ++kk) {
        // A[m][k=v] = Lhs[v][m]: trans load of Lhs rows v (16 x 16 block at rows kk*16.., cols m0..)
        uint32_t a[4];
        {
          const int vr = kk * 16 + (lane & 7) + ((lane >> 4) << 3);
          const int mc = m0 + (((lane >> 3) & 1) << 3);
          ldsm_x4_t(a, smem_u32(Lhs + swz(vr, mc >> 3)));
        }
#pragma unroll
        for (int i2 = 0; i2 < 4; ++i2) {
          // B[k=v][n] = Rhs[v][n]: trans load
          uint32_t b[4];
          const int vr = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
          const int c = i2 * 2 + (lane >> 4);
          ldsm_x4_t(b, smem_u32(Rhs + swz(vr, c)));
          mma16816(wacc[2 * i2], a, b[0], b[1]);
          mma16816(wacc[2 * i2 + 1], a, b[2], b[3]);
        }
      }
      __syncthreads();
    }
  }
  // flush the reductions
  if (ds_in_regs) {
    const int h = g % p.H;
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int e2 = 0; e2 < 2; ++e2) {
        const int d = i * 8 + cc + e2;
        if (d < p.D) atomicAdd(&gsm[h * 64 + d], dsacc[i][e2]);
      }
  }
  __syncthreads();
  if (p.gate) {
    const int m0 = (warp & 3) * 16;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int m = m0 + g + (e >> 1) * 8;
        const int n = i * 8 + cc + (e & 1);
        if (warp < 4) {  // dW2 [D, 64]: m = d, n = j
          if (m < p.D) atomicAdd(&p.gw2[m * 64 + n], wacc[i][e]);
        } else {  // dW1 [64, D]: m = j, n = d
          if (n < p.D) atomicAdd(&p.gw1[m * p.D + n], wacc[i][e]);
        }
      }
    }
    for (int i = threadIdx.x; i < 64; i += blockDim.x) {
      atomicAdd(&p.gb1[i], gb1[i]);
      if (i < p.D) atomicAdd(&p.gb2[i], gb2[i]);
    }
  }
  for (int i = threadIdx.x; i < p.H * 64; i += blockDim.x) {
    const int h = i >> 6, d = i & 63;
    if (d < p.D) atomicAdd(&p.gs[h * p.D + d], gsm[i]);
  }
}

}  // namespace qass

// tensor-core kernels (qass_tc.cu)
bool qass_tc_supported(int64_t H, int64_t D);
void qass_tc_launch(bool bwd, const torch::Tensor& q, const torch::Tensor* dout, torch::Tensor& out,
                    const float* s, const float* w1, const float* b1, const float* w2, const float* b2, float* gs,
                    float* gw1, float* gb1, float* gw2, float* gb2, int64_t H, int64_t D, int* status);

static int* opt_status(const c10::optional<torch::Tensor>& st) {
  if (!st.has_value() || !st->defined()) return nullptr;
  TORCH_CHECK(st->is_cuda() && st->scalar_type() == at::kInt && st->numel() >= 1, "qass: int32 status word");
  return st->data_ptr<int>();
}

static int sm_count(int dev) {
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

static void check_q(const torch::Tensor& q, int64_t H, int64_t D) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && q.dim() == 2 && q.stride(1) == 1,
              "qass: bf16 [R, >= H*D] row-major q");
  TORCH_CHECK(D > 0 && D <= 64 && D % 8 == 0 && q.size(1) >= H * D, "qass: head dim multiple of 8, <= 64");
  TORCH_CHECK(q.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0, "qass: 16-byte rows");
  TORCH_CHECK(q.size(0) * H < 2147483647LL, "qass: at most 2^31 - 1 (row, head) vectors per call");
}

// q' = q * s * (1 + tanh(gate(q))) (gate optional) -> new [R, H*D] bf16
torch::Tensor qass_fwd(const torch::Tensor& q, const torch::Tensor& s, const c10::optional<torch::Tensor>& w1,
                       const c10::optional<torch::Tensor>& b1, const c10::optional<torch::Tensor>& w2,
                       const c10::optional<torch::Tensor>& b2, int64_t H, int64_t D,
                       const c10::optional<torch::Tensor>& status) {
  check_q(q, H, D);
  const at::cuda::CUDAGuard guard(q.device());
  auto out = torch::empty({q.size(0), H * D}, q.options());
  qass::Params p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.ldq = q.stride(0);
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ldo = out.stride(0);
  auto sc = s.contiguous().to(torch::kFloat);
  p.s = sc.data_ptr<float>();
  p.gate = w1.has_value() && w1->defined();
  torch::Tensor w1c, b1c, w2c, b2c;
  if (p.gate) {
    w1c = w1->contiguous().to(torch::kFloat);
    b1c = b1->contiguous().to(torch::kFloat);
    w2c = w2->contiguous().to(torch::kFloat);
    b2c = b2->contiguous().to(torch::kFloat);
    TORCH_CHECK(w1c.size(0) == 64 && w1c.size(1) == D && w2c.size(0) == D && w2c.size(1) == 64,
                "qass: gate MLP must be D -> 64 -> D");
    p.w1 = w1c.data_ptr<float>();
    p.b1 = b1c.data_ptr<float>();
    p.w2 = w2c.data_ptr<float>();
    p.b2 = b2c.data_ptr<float>();
  }
  p.R = q.size(0);
  p.H = static_cast<int>(H);
  p.D = static_cast<int>(D);
  if (p.R == 0) return out;
  if (p.gate && qass_tc_supported(H, D)) {
    qass_tc_launch(false, q, nullptr, out, p.s, p.w1, p.b1, p.w2, p.b2, nullptr, nullptr, nullptr, nullptr, nullptr,
                   H, D, opt_status(status));
    return out;
  }
  if (!p.gate) {
    // the gate-free path still stages (zero) weights: give it valid pointers
    w1c = torch::zeros({64, D}, q.options().dtype(torch::kFloat));
    w2c = torch::zeros({D, 64}, q.options().dtype(torch::kFloat));
    p.w1 = w1c.data_ptr<float>();
    p.w2 = w2c.data_ptr<float>();
  }
  const int64_t groups = (p.R * p.H + qass::kVec - 1) / qass::kVec;
  const int blocks = static_cast<int>(std::min<int64_t>((groups + qass::kWarps - 1) / qass::kWarps, sm_count(q.get_device()) * 8));
  const int dynf = qass::kWarps * 2 * 16 * 128 + static_cast<int>(H) * 64 * static_cast<int>(sizeof(float));
  static int fwd_smem_set[64] = {0};  // once per device (and whenever a larger size is needed)
  const int dev = q.get_device();
  if (fwd_smem_set[dev] < dynf) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(qass::qass_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dynf));
    fwd_smem_set[dev] = dynf;
  }
  qass::qass_fwd_kernel<<<blocks, qass::kThreads, dynf, at::cuda::getCurrentCUDAStream()>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

// Backward: returns dq (bf16 [R, H*D]) and fills ds / dW1 / db1 / dW2 / db2 (fp32, zeroed by the caller).
torch::Tensor qass_bwd(const torch::Tensor& q, const torch::Tensor& dout, const torch::Tensor& s,
                       const c10::optional<torch::Tensor>& w1, const c10::optional<torch::Tensor>& b1,
                       const c10::optional<torch::Tensor>& w2, const c10::optional<torch::Tensor>& b2,
                       torch::Tensor& gs, const c10::optional<torch::Tensor>& gw1,
                       const c10::optional<torch::Tensor>& gb1, const c10::optional<torch::Tensor>& gw2,
                       const c10::optional<torch::Tensor>& gb2, int64_t H, int64_t D,
                       const c10::optional<torch::Tensor>& out, const c10::optional<torch::Tensor>& status) {
  check_q(q, H, D);
  TORCH_CHECK(dout.scalar_type() == at::kFloat && dout.dim() == 2 && dout.stride(1) == 1 && dout.size(0) == q.size(0),
              "qass_bwd: fp32 [R, H*D] gradient");
  TORCH_CHECK(gs.scalar_type() == at::kFloat && gs.is_contiguous() && gs.numel() == H * D, "qass_bwd: ds [H, D]");
  TORCH_CHECK(dout.stride(0) % 4 == 0 && reinterpret_cast<uintptr_t>(dout.data_ptr()) % 16 == 0,
              "qass_bwd: gradient rows must be 16-byte aligned");
  const at::cuda::CUDAGuard guard(q.device());
  torch::Tensor dq;
  if (out.has_value() && out->defined()) {  // written in place (e.g. a column block of a wider gradient)
    dq = *out;
    TORCH_CHECK(dq.scalar_type() == at::kBFloat16 && dq.dim() == 2 && dq.size(0) == q.size(0) &&
                    dq.size(1) == H * D && dq.stride(1) == 1 && dq.stride(0) % 2 == 0 &&
                    reinterpret_cast<uintptr_t>(dq.data_ptr()) % 4 == 0,
                "qass_bwd: out must be bf16 [R, H*D] with unit column stride and 4-byte aligned rows");
  } else {
    dq = torch::empty({q.size(0), H * D}, q.options());
  }
  qass::Params p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.ldq = q.stride(0);
  p.out = reinterpret_cast<__nv_bfloat16*>(dq.data_ptr());
  p.ldo = dq.stride(0);
  p.dout = dout.data_ptr<float>();
  p.ldd = dout.stride(0);
  auto sc = s.contiguous().to(torch::kFloat);
  p.s = sc.data_ptr<float>();
  p.gs = gs.data_ptr<float>();
  p.gate = w1.has_value() && w1->defined();
  torch::Tensor w1c, b1c, w2c, b2c;
  if (p.gate) {
    w1c = w1->contiguous().to(torch::kFloat);
    b1c = b1->contiguous().to(torch::kFloat);
    w2c = w2->contiguous().to(torch::kFloat);
    b2c = b2->contiguous().to(torch::kFloat);
    p.w1 = w1c.data_ptr<float>();
    p.b1 = b1c.data_ptr<float>();
    p.w2 = w2c.data_ptr<float>();
    p.b2 = b2c.data_ptr<float>();
    for (const auto* t : {&gw1, &gb1, &gw2, &gb2})
      TORCH_CHECK(t->has_value() && (*t)->scalar_type() == at::kFloat && (*t)->is_contiguous(),
                  "qass_bwd: fp32 weight-gradient accumulators");
    p.gw1 = gw1->data_ptr<float>();
    p.gb1 = gb1->data_ptr<float>();
    p.gw2 = gw2->data_ptr<float>();
    p.gb2 = gb2->data_ptr<float>();
  } else {
    w1c = torch::zeros({64, D}, q.options().dtype(torch::kFloat));
    w2c = torch::zeros({D, 64}, q.options().dtype(torch::kFloat));
    p.w1 = w1c.data_ptr<float>();
    p.w2 = w2c.data_ptr<float>();
  }
  p.R = q.size(0);
  p.H = static_cast<int>(H);
  p.D = static_cast<int>(D);
  if (p.R == 0) return dq;
  if (p.gate && qass_tc_supported(H, D)) {
    TORCH_CHECK(reinterpret_cast<uintptr_t>(dq.data_ptr()) % 16 == 0 && dq.stride(0) % 8 == 0,
                "qass_bwd: the tensor-core kernel writes 16-byte row chunks of dq");
    TORCH_CHECK(gb2->numel() >= D && gb1->numel() >= 64 && gw1->numel() >= 64 * D && gw2->numel() >= D * 64,
                "qass_bwd: weight-gradient accumulator shapes");
    qass_tc_launch(true, q, &dout, dq, p.s, p.w1, p.b1, p.w2, p.b2, p.gs, p.gw1, p.gb1, p.gw2, p.gb2, H, D,
                   opt_status(status));
    return dq;
  }
  const int64_t steps = (p.R * p.H + qass::kStageVec - 1) / qass::kStageVec;
  const int blocks = static_cast<int>(std::min<int64_t>(steps, sm_count(q.get_device()) * 2));
  const int dyn = 4 * qass::kStageVec * 128 + qass::kWarps * 2 * 16 * 128 +
                  qass::kWarps * 2 * 16 * qass::kDoutLd * static_cast<int>(sizeof(float)) +
                  2 * static_cast<int>(H) * 64 * static_cast<int>(sizeof(float));
  static int bwd_smem_set[64] = {0};
  const int dev = q.get_device();
  if (bwd_smem_set[dev] < dyn) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(qass::qass_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn));
    bwd_smem_set[dev] = dyn;
  }
  qass::qass_bwd_kernel<<<blocks, qass::kThreads, dyn, at::cuda::getCurrentCUDAStream()>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dq;
}

}  // namespace nori
