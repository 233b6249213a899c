// Query-aware scalable softmax (QASS) gate on the 5th-generation tensor cores.
//
//   q' = q * s[h] * (1 + tanh(W2 gelu(W1 q + b1) + b2))        (reference
//   model/layer.py:316-456, mode "full")
//
// One tile = 128 query vectors (token row x head, in memory order).  Per tile:
//
//   TMA      q tile [128 x 64] bf16 (3-D map {D, H, R}: columns >= D and rows >= R are
//            zero-filled), and for the backward the fp32 incoming gradient in two
//            [128 x 32] halves, all 128-byte swizzled;
//   tcgen05  z1 = q W1^T, z2 = gelu(z1) W2^T (M = 128 vectors, N = K = 64, fp32
//            accumulators in TMEM); the backward adds dG = dz2 W2, dq_mlp = dz1 W1 (W read
//            MN-major) and, accumulated across all tiles of the CTA, the weight and bias
//            gradients as ONE M = 128 product  [dz2^T; dz1^T] x [q | G]  (the diagonal
//            blocks are dW2 and dW1; the shared-memory tiles written for the forward
//            products are read MN-major here), the bias sums as [dz2^T; dz1^T] x 1 and
//            the per-head base-scale gradient as X^T x onehot(head) with
//            X = dq' (1 + tanh) q;
//   epilogue one thread per vector (TMEM lane = vector): GELU / GELU' / tanh arithmetic,
//            the bf16 operand tiles for the next product, the output row.
//
// Warp roles: warps 0-7 are two epilogue warpgroups, each owning one of two tile slots
// (shared memory + TMEM columns) so that two tiles are in flight; warp 8 issues the TMA
// loads, warp 9 owns TMEM and issues every MMA from a polling state machine over both
// slots.  All waits are bounded (status word + abort flag, no trap).
//
// TMEM columns: slot s: [128 s, 128 s + 64) z1 -> GELU'(z1) -> dq_mlp, [128 s + 64,
// 128 s + 128) z2 -> dG; backward accumulators: 256..383 [dz2^T; dz1^T] [q | G],
// 384..399 bias sums, 400..415 base-scale sums.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "sm100.cuh"
#include "tma_host.h"

namespace nori {
namespace qtc {

constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 10 * 32;
constexpr int kSRow = 68;   // fp32 stride of one head's base-scale row (spreads heads over banks)
constexpr int kMaxHeads = 16;

// barrier indices (per slot s: index + s); the forward's q tiles arrive through a ring of
// kRing stages of their own (kRingFull / kRingEmpty + stage), so the loads run several
// tiles ahead of the two compute slots
constexpr int kRing = 6;
enum : int { kLoad = 0, kMma1 = 2, kGReady = 4, kMma2 = 6, kDz2 = 8, kMma3 = 10, kDz1 = 12, kMma4 = 14,
             kTFree = 16, kAcc = 18, kRingFull = 19, kRingEmpty = kRingFull + kRing, kNumBars = kRingEmpty + kRing };

template <bool BWD>
struct Lay {
  static constexpr int kW1 = 0, kW2 = 8192, kOneHot = 16384, kOnes = 20480, kSlot0 = 24576;
  static constexpr int kQ = 0, kG = 16384, kDz2 = 32768, kDz1 = 49152, kDout = 65536;  // within a slot
  // forward: the slots hold only their G tile; q tiles sit in the ring after them
  static constexpr int kSlotBytes = BWD ? 98304 : 32768;
  static constexpr int kRing0 = kSlot0 + 2 * kSlotBytes;
  static constexpr int kRingBytes = BWD ? 0 : kRing * 16384;
  static constexpr int kB1 = kRing0 + kRingBytes;
  static constexpr int kB2 = kB1 + 256;
  static constexpr int kS = kB2 + 256;
  static constexpr int kBar = kS + kMaxHeads * kSRow * 4;
  static constexpr int kTmemPtr = kBar + kNumBars * 8;
  static constexpr int kBytes = kTmemPtr + 16;
  static constexpr int kAlloc = kBytes + 1024;  // slack for aligning the base to 1024 bytes
  static constexpr uint32_t kTmemCols = BWD ? 512 : 256;
};

struct Params {
  int64_t nvec;  // R * H
  int H, D;
  __nv_bfloat16* out;
  int64_t ldo;
  const float* w1;  // [64, D]
  const float* b1;  // [64]
  const float* w2;  // [D, 64]
  const float* b2;  // [D]
  const float* s;   // [H, D]
  float* gw1;
  float* gb1;
  float* gw2;
  float* gb2;
  float* gs;
  int* status;
};

// byte offset of 16-byte chunk `c` of row `r` in a 128-byte-swizzled tile of 128-byte rows
__device__ __forceinline__ uint32_t sw(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

// The gate's activations cost one MUFU instruction each (tanh.approx.f32, max relative error
// about 2^-11): GELU in its tanh form, 0.5 z (1 + tanh(c (z + 0.044715 z^3))) with
// c = sqrt(2 / pi) (Hendrycks & Gimpel 2016; within 2e-4 of the erf form, far below the bf16
// rounding of q'), its derivative taken from the same form, and the gate's tanh itself. The
// erf / exp / divide forms took two to three MUFU operations per element and bound the epilogue.
__device__ __forceinline__ float tanh_mufu(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float kGeluC = 0.7978845608028654f;  // sqrt(2 / pi)
constexpr float kGeluA = 0.044715f;
__device__ __forceinline__ float gelu_f(float z) {
  const float t = tanh_mufu(kGeluC * fmaf(kGeluA * z * z, z, z));
  const float h = 0.5f * z;
  return fmaf(h, t, h);
}
__device__ __forceinline__ void gelu_grad(float z, float& g, float& dg) {
  const float z2 = z * z;
  const float t = tanh_mufu(kGeluC * fmaf(kGeluA * z2, z, z));
  const float cdf = fmaf(0.5f, t, 0.5f);
  g = z * cdf;
  // d/dz of 0.5 z (1 + t): 0.5 (1 + t) + 0.5 z (1 - t^2) c (1 + 3 a z^2)
  dg = fmaf(0.5f * z * fmaf(-t, t, 1.0f), kGeluC * fmaf(3.0f * kGeluA, z2, 1.0f), cdf);
}
__device__ __forceinline__ float tanh_fast(float x) { return tanh_mufu(x); }

// 32 consecutive bf16 values of row `r`, starting at column 32 c, of a swizzled tile
__device__ __forceinline__ void load_row32_bf16(uint32_t tile, int r, int c, uint32_t (&w)[16]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint4 v = ld_shared_v4(tile + sw(r, 4 * c + j));
    w[4 * j] = v.x;
    w[4 * j + 1] = v.y;
    w[4 * j + 2] = v.z;
    w[4 * j + 3] = v.w;
  }
}
__device__ __forceinline__ void store_row32_bf16(uint32_t tile, int r, int c, const uint32_t (&w)[16]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) st_shared_v4(tile + sw(r, 4 * c + j), w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
}

// One output row (D bf16 values, 32 per call) to global memory.
__device__ __forceinline__ void store_out32(__nv_bfloat16* dst, int c, int D, const uint32_t (&w)[16]) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
    if (32 * c + 8 * j < D)
      *reinterpret_cast<uint4*>(dst + 32 * c + 8 * j) = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
}

template <bool BWD>
__global__ void __launch_bounds__(kThreads, 1)
    qass_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmdo, Params p) {
  using L = Lay<BWD>;
  extern __shared__ uint8_t qtc_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(qtc_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(sm);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L::kBar);
  uint32_t* tmem_ptr = reinterpret_cast<uint32_t*>(sm + L::kTmemPtr);
  float* sb1 = reinterpret_cast<float*>(sm + L::kB1);
  float* sb2 = reinterpret_cast<float*>(sm + L::kB2);
  float* ss = reinterpret_cast<float*>(sm + L::kS);
  __shared__ int abort_flag;
  volatile int* abort = &abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = p.H, D = p.D;
  const int64_t ntiles = (p.nvec + 127) / 128;
  const int my_tiles = ntiles > blockIdx.x ? static_cast<int>((ntiles - 1 - blockIdx.x) / gridDim.x + 1) : 0;

  // ---- prologue: weights (bf16, swizzled, zero padded), constants, barriers, TMEM
  for (int i = threadIdx.x; i < 64 * 64; i += blockDim.x) {
    const int r = i >> 6, c = i & 63;
    const float w1 = c < D ? p.w1[r * D + c] : 0.f;  // W1 rows = hidden j, cols = dim d
    const float w2 = r < D ? p.w2[r * 64 + c] : 0.f;  // W2 rows = dim d, cols = hidden j
    reinterpret_cast<__nv_bfloat16*>(sm + L::kW1 + sw(r, c >> 3))[c & 7] = __float2bfloat16(w1);
    reinterpret_cast<__nv_bfloat16*>(sm + L::kW2 + sw(r, c >> 3))[c & 7] = __float2bfloat16(w2);
  }
  if (BWD) {
    // one-hot head matrix [16 rows h x 128 vectors], K-major, two 64-column atoms
    for (int i = threadIdx.x; i < 16 * 128; i += blockDim.x) {
      const int h = i >> 7, v = i & 127;
      const int atom = v >> 6, col = v & 63;
      const float x = (h < H && v % H == h) ? 1.f : 0.f;
      reinterpret_cast<__nv_bfloat16*>(sm + L::kOneHot + atom * 2048 + sw(h, col >> 3))[col & 7] = __float2bfloat16(x);
    }
    for (int i = threadIdx.x; i < 16 * 64; i += blockDim.x)
      reinterpret_cast<__nv_bfloat16*>(sm + L::kOnes)[i] = __float2bfloat16(1.f);
  }
  for (int i = threadIdx.x; i < 64; i += blockDim.x) {
    sb1[i] = p.b1[i];
    sb2[i] = i < D ? p.b2[i] : 0.f;
  }
  for (int i = threadIdx.x; i < kMaxHeads * kSRow; i += blockDim.x) {
    const int h = i / kSRow, d = i % kSRow;
    ss[i] = (h < H && d < D) ? p.s[h * D + d] : 0.f;
  }
  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar[kLoad + s], 1);
      mbar_init(&bar[kMma1 + s], 1);
      mbar_init(&bar[kGReady + s], 128);
      mbar_init(&bar[kMma2 + s], 1);
      mbar_init(&bar[kDz2 + s], 128);
      mbar_init(&bar[kMma3 + s], 1);
      mbar_init(&bar[kDz1 + s], 128);
      mbar_init(&bar[kMma4 + s], 1);
      mbar_init(&bar[kTFree + s], 128);
    }
    for (int i = 0; i < kRing; ++i) {
      mbar_init(&bar[kRingFull + i], 1);
      mbar_init(&bar[kRingEmpty + i], 128);  // the epilogue warpgroup that used the tile
    }
    mbar_init(&bar[kAcc], 1);
    fence_barrier_init();
  }
  if (warp == kMmaWarp) tmem_alloc(tmem_ptr, L::kTmemCols);
  fence_proxy_async_smem();  // the staged weights are read by the tensor cores (async proxy)
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_ptr;

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ TMA producer
    if (!BWD && elect_one()) {
      for (int i = 0; i < my_tiles; ++i) {
        const int st = i % kRing;
        if (!mbar_wait(&bar[kRingEmpty + st], ((i / kRing) & 1) ^ 1, p.status, kTimeoutProducer, abort)) break;
        const int64_t tile = blockIdx.x + static_cast<int64_t>(i) * gridDim.x;
        const int r0 = static_cast<int>(tile * 128 / H);
        mbar_arrive_expect_tx(&bar[kRingFull + st], 16384);
        tma_load_3d(sm + L::kRing0 + st * 16384, &tmq, &bar[kRingFull + st], 0, 0, r0);
      }
      // never leave with copies in flight: wait (bounded, ignoring aborts) for the last ones
      for (int i = my_tiles > kRing ? my_tiles - kRing : 0; i < my_tiles; ++i)
        mbar_wait(&bar[kRingFull + i % kRing], static_cast<uint32_t>(i / kRing) & 1, nullptr, 0, nullptr);
    } else if (BWD && elect_one()) {
      int issued[2] = {-1, -1};
      for (int i = 0; i < my_tiles; ++i) {
        const int s = i & 1;
        const uint32_t n = static_cast<uint32_t>(i >> 1);
        if (!mbar_wait(&bar[kTFree + s], (n & 1) ^ 1, p.status, kTimeoutProducer, abort)) break;
        const int64_t tile = blockIdx.x + static_cast<int64_t>(i) * gridDim.x;
        const int r0 = static_cast<int>(tile * 128 / H);
        uint8_t* slot = sm + L::kSlot0 + s * L::kSlotBytes;
        mbar_arrive_expect_tx(&bar[kLoad + s], BWD ? 16384 + 32768 : 16384);
        tma_load_3d(slot + L::kQ, &tmq, &bar[kLoad + s], 0, 0, r0);
        if (BWD) {
          tma_load_3d(slot + L::kDout, &tmdo, &bar[kLoad + s], 0, 0, r0);
          tma_load_3d(slot + L::kDout + 16384, &tmdo, &bar[kLoad + s], 32, 0, r0);
        }
        issued[s] = static_cast<int>(n);
      }
      // never leave with copies in flight: wait (bounded, ignoring aborts) for the last ones
      for (int s = 0; s < 2; ++s)
        if (issued[s] >= 0) mbar_wait(&bar[kLoad + s], static_cast<uint32_t>(issued[s]) & 1, nullptr, 0, nullptr);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t id_kk = umma_idesc_bf16(128, 64, false, false);
      constexpr uint32_t id_kn = umma_idesc_bf16(128, 64, false, true);
      constexpr uint32_t id_w = umma_idesc_bf16(128, 128, true, true);
      constexpr uint32_t id_b = umma_idesc_bf16(128, 16, true, false);
      const uint32_t w1 = sbase + L::kW1, w2 = sbase + L::kW2;
      int state[2] = {0, 0};
      int idx[2] = {0, 1};
      int remaining = my_tiles;
      bool acc_started = false;
      uint64_t t_last = globaltimer_ns();
      uint32_t spins = 0;
      while (remaining > 0) {
        bool progressed = false;
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          const int i = idx[s];
          if (i >= my_tiles) continue;
          const uint32_t par = static_cast<uint32_t>(i >> 1) & 1;
          const uint32_t slot = sbase + L::kSlot0 + s * L::kSlotBytes;
          const uint32_t tA = tmem + s * 128, tB = tA + 64;
          if (state[s] == 0) {
            const uint32_t qt = BWD ? slot + L::kQ : sbase + L::kRing0 + (i % kRing) * 16384;
            if (BWD ? !mbar_try_wait(&bar[kLoad + s], par)
                    : !mbar_try_wait(&bar[kRingFull + i % kRing], static_cast<uint32_t>(i / kRing) & 1))
              continue;
            tc_fence_after();
#pragma unroll
            for (int k = 0; k < 4; ++k)
              umma_bf16_ss(tA, umma_desc_kmajor_sw128(qt + k * 32), umma_desc_kmajor_sw128(w1 + k * 32),
                           id_kk, k > 0);
            umma_commit(&bar[kMma1 + s]);
            state[s] = 1;
          } else if (state[s] == 1) {
            if (!mbar_try_wait(&bar[kGReady + s], par)) continue;
            tc_fence_after();
#pragma unroll
            for (int k = 0; k < 4; ++k)
              umma_bf16_ss(tB, umma_desc_kmajor_sw128(slot + L::kG + k * 32), umma_desc_kmajor_sw128(w2 + k * 32),
                           id_kk, k > 0);
            umma_commit(&bar[kMma2 + s]);
            if (BWD) {
              state[s] = 2;
            } else {
              state[s] = 0;
              idx[s] += 2;
              --remaining;
            }
          } else if (state[s] == 2) {
            if (!mbar_try_wait(&bar[kDz2 + s], par)) continue;
            tc_fence_after();
            // dG[v][j] = sum_d dz2[v][d] W2[d][j]: W2 tile rows are K (d), N (j) contiguous
#pragma unroll
            for (int k = 0; k < 4; ++k)
              umma_bf16_ss(tB, umma_desc_kmajor_sw128(slot + L::kDz2 + k * 32),
                           umma_smem_desc(w2 + k * 2048, 16384, 1024, 2), id_kn, k > 0);
            umma_commit(&bar[kMma3 + s]);
            state[s] = 3;
          } else {
            if (!mbar_try_wait(&bar[kDz1 + s], par)) continue;
            tc_fence_after();
            // dq_mlp[v][d] = sum_j dz1[v][j] W1[j][d]  (into the z1 / GELU' columns, now free)
#pragma unroll
            for (int k = 0; k < 4; ++k)
              umma_bf16_ss(tA, umma_desc_kmajor_sw128(slot + L::kDz1 + k * 32),
                           umma_smem_desc(w1 + k * 2048, 16384, 1024, 2), id_kn, k > 0);
            // [dz2^T; dz1^T] (M = 128: d then j) x [q | G] (N = 128), K = the 128 vectors
#pragma unroll
            for (int k = 0; k < 8; ++k)
              umma_bf16_ss(tmem + 256, umma_smem_desc(slot + L::kDz2 + k * 2048, 16384, 1024, 2),
                           umma_smem_desc(slot + L::kQ + k * 2048, 16384, 1024, 2), id_w, acc_started || k > 0);
            // bias sums: [dz2^T; dz1^T] x ones
#pragma unroll
            for (int k = 0; k < 8; ++k)
              umma_bf16_ss(tmem + 384, umma_smem_desc(slot + L::kDz2 + k * 2048, 16384, 1024, 2),
                           umma_desc_kmajor_sw128(sbase + L::kOnes + (k & 3) * 32), id_b, acc_started || k > 0);
            // base-scale sums per head: X^T x onehot (rows 64..127 of this product are unused)
#pragma unroll
            for (int k = 0; k < 8; ++k)
              umma_bf16_ss(tmem + 400, umma_smem_desc(slot + L::kDout + k * 2048, 16384, 1024, 2),
                           umma_desc_kmajor_sw128(sbase + L::kOneHot + (k >> 2) * 2048 + (k & 3) * 32), id_b,
                           acc_started || k > 0);
            acc_started = true;
            umma_commit(&bar[kMma4 + s]);
            state[s] = 0;
            idx[s] += 2;
            --remaining;
          }
          progressed = true;
        }
        if (progressed) {
          spins = 0;
          t_last = globaltimer_ns();
        } else if ((++spins & 255u) == 0) {
          if (*abort) break;
          if (globaltimer_ns() - t_last > kWaitLimitNs) {
            record_status(p.status, kTimeoutMma);
            *abort = 1;
            break;
          }
        }
      }
      umma_commit(&bar[kAcc]);  // arrives once every MMA issued above has completed
    }
  } else {
    // ------------------------------------------------------------ epilogue warpgroups
    const int s = warp >> 2;
    const int lb = (warp & 3) * 32;
    const int r = lb + lane;  // vector within the tile = TMEM lane
    const int h = r % H;      // 128 % H == 0: the head of a tile row never changes
    const uint32_t slot = sbase + L::kSlot0 + s * L::kSlotBytes;
    const uint32_t tA = tmem + (static_cast<uint32_t>(lb) << 16) + s * 128, tB = tA + 64;
    const float* srow = ss + h * kSRow;
    bool ok = true;
    for (int i = s; i < my_tiles && ok; i += 2) {
      const uint32_t par = static_cast<uint32_t>(i >> 1) & 1;
      const int64_t v = (blockIdx.x + static_cast<int64_t>(i) * gridDim.x) * 128 + r;
      const bool valid = v < p.nvec;
      __nv_bfloat16* dst = nullptr;
      if (valid) {
        const uint32_t vv = static_cast<uint32_t>(v);
        const uint32_t row = vv / static_cast<uint32_t>(H);
        dst = p.out + static_cast<int64_t>(row) * p.ldo + static_cast<int64_t>(vv - row * H) * D;
      }
      // phase 1: z1 -> G (bf16 operand tile) [and GELU'(z1) back into TMEM]
      if (!mbar_wait_warp(&bar[kMma1 + s], par, p.status, kTimeoutEpilogue, abort)) { ok = false; break; }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t z[32];
        tmem_ld32(tA + 32 * c, z);
        tmem_wait_ld();
        uint32_t gw[16];
#pragma unroll
        for (int k = 0; k < 32; k += 2) {
          float g0, g1;
          if (BWD) {
            float d0, d1;
            gelu_grad(__uint_as_float(z[k]) + sb1[32 * c + k], g0, d0);
            gelu_grad(__uint_as_float(z[k + 1]) + sb1[32 * c + k + 1], g1, d1);
            z[k] = __float_as_uint(d0);
            z[k + 1] = __float_as_uint(d1);
          } else {
            g0 = gelu_f(__uint_as_float(z[k]) + sb1[32 * c + k]);
            g1 = gelu_f(__uint_as_float(z[k + 1]) + sb1[32 * c + k + 1]);
          }
          gw[k >> 1] = pack_bf16x2(g0, g1);
        }
        store_row32_bf16(slot + L::kG, r, c, gw);
        if (BWD) tmem_st32(tA + 32 * c, z);
      }
      if (BWD) tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bar[kGReady + s]);
      // phase 2: z2 -> output (forward) or dz2, X and the direct part of dq (backward)
      if (!mbar_wait_warp(&bar[kMma2 + s], par, p.status, kTimeoutEpilogue, abort)) { ok = false; break; }
      const uint32_t qtile = BWD ? slot + L::kQ : sbase + L::kRing0 + (i % kRing) * 16384;
      if (BWD ? !mbar_wait_warp(&bar[kLoad + s], par, p.status, kTimeoutEpilogue, abort)
              : !mbar_wait_warp(&bar[kRingFull + i % kRing], static_cast<uint32_t>(i / kRing) & 1, p.status,
                                kTimeoutEpilogue, abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float dqd[2][32];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t z[32];
        tmem_ld32(tB + 32 * c, z);
        uint32_t qw[16];
        load_row32_bf16(qtile, r, c, qw);
        tmem_wait_ld();
        if (!BWD) {
          uint32_t ow[16];
#pragma unroll
          for (int k = 0; k < 32; k += 2) {
            const int d = 32 * c + k;
            const float t0 = tanh_fast(__uint_as_float(z[k]) + sb2[d]);
            const float t1 = tanh_fast(__uint_as_float(z[k + 1]) + sb2[d + 1]);
            ow[k >> 1] = pack_bf16x2(bf16lo(qw[k >> 1]) * srow[d] * (1.f + t0),
                                     bf16hi(qw[k >> 1]) * srow[d + 1] * (1.f + t1));
          }
          if (valid) store_out32(dst, c, D, ow);
        } else {
          float go[32];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint4 w = ld_shared_v4(slot + L::kDout + c * 16384 + sw(r, j));
            go[4 * j] = __uint_as_float(w.x);
            go[4 * j + 1] = __uint_as_float(w.y);
            go[4 * j + 2] = __uint_as_float(w.z);
            go[4 * j + 3] = __uint_as_float(w.w);
          }
          uint32_t xw[16], zw[16];
#pragma unroll
          for (int k = 0; k < 32; k += 2) {
            float xo[2], zo[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int d = 32 * c + k + e;
              const float t = tanh_fast(__uint_as_float(z[k + e]) + sb2[d]);
              const float gate = 1.f + t;
              const float x = e ? bf16hi(qw[k >> 1]) : bf16lo(qw[k >> 1]);
              const float sv = srow[d];
              const float dq_ = go[k + e];
              dqd[c][k + e] = dq_ * gate * sv;
              xo[e] = dq_ * gate * x;
              zo[e] = dq_ * x * sv * (1.f - t * t);
            }
            xw[k >> 1] = pack_bf16x2(xo[0], xo[1]);
            zw[k >> 1] = pack_bf16x2(zo[0], zo[1]);
          }
          // X overwrites this row of the (already read) first gradient half
          store_row32_bf16(slot + L::kDout, r, c, xw);
          store_row32_bf16(slot + L::kDz2, r, c, zw);
        }
      }
      if (!BWD) {
        tc_fence_before();
        mbar_arrive(&bar[kRingEmpty + i % kRing]);  // the q tile's stage may be refilled
        continue;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bar[kDz2 + s]);
      // phase 3: dz1 = dG * GELU'(z1)
      if (!mbar_wait_warp(&bar[kMma3 + s], par, p.status, kTimeoutEpilogue, abort)) { ok = false; break; }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t dg[32], gp[32];
        tmem_ld32(tB + 32 * c, dg);
        tmem_ld32(tA + 32 * c, gp);
        tmem_wait_ld();
        uint32_t w[16];
#pragma unroll
        for (int k = 0; k < 32; k += 2)
          w[k >> 1] = pack_bf16x2(__uint_as_float(dg[k]) * __uint_as_float(gp[k]),
                                  __uint_as_float(dg[k + 1]) * __uint_as_float(gp[k + 1]));
        store_row32_bf16(slot + L::kDz1, r, c, w);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bar[kDz1 + s]);
      // phase 4: dq = direct part + dz1 W1
      if (!mbar_wait_warp(&bar[kMma4 + s], par, p.status, kTimeoutEpilogue, abort)) { ok = false; break; }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t m[32];
        tmem_ld32(tA + 32 * c, m);
        tmem_wait_ld();
        uint32_t w[16];
#pragma unroll
        for (int k = 0; k < 32; k += 2)
          w[k >> 1] = pack_bf16x2(dqd[c][k] + __uint_as_float(m[k]), dqd[c][k + 1] + __uint_as_float(m[k + 1]));
        if (valid) store_out32(dst, c, D, w);
      }
      tc_fence_before();
      mbar_arrive(&bar[kTFree + s]);
    }
    if (BWD && s == 0 && ok && my_tiles > 0) {
      // flush the CTA's gradient accumulators (lane = row of the stacked product)
      if (mbar_wait_warp(&bar[kAcc], 0, p.status, kTimeoutEpilogue, abort)) {
        tc_fence_after();
        const uint32_t tl = tmem + (static_cast<uint32_t>(lb) << 16);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t a[32];
          tmem_ld32(tl + 256 + (r < 64 ? 64 : 0) + 32 * c, a);  // uniform per warp (lanes 0-63 / 64-127)
          tmem_wait_ld();
          if (r < 64) {  // dW2[d][j], d = r
            if (r < D)
#pragma unroll
              for (int k = 0; k < 32; ++k) atomicAdd(&p.gw2[r * 64 + 32 * c + k], __uint_as_float(a[k]));
          } else {  // dW1[j][d], j = r - 64
#pragma unroll
            for (int k = 0; k < 32; ++k)
              if (32 * c + k < D) atomicAdd(&p.gw1[(r - 64) * D + 32 * c + k], __uint_as_float(a[k]));
          }
        }
        uint32_t bsum[16], hsum[16];
        tmem_ld16(tl + 384, bsum);
        tmem_ld16(tl + 400, hsum);
        tmem_wait_ld();
        if (r < 64) {
          if (r < D) {
            atomicAdd(&p.gb2[r], __uint_as_float(bsum[0]));
            for (int hh = 0; hh < H; ++hh) atomicAdd(&p.gs[hh * D + r], __uint_as_float(hsum[hh]));
          }
        } else {
          atomicAdd(&p.gb1[r - 64], __uint_as_float(bsum[0]));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    // the final commit covers every MMA this CTA issued: wait for it (bounded) before freeing TMEM
    mbar_wait_warp(&bar[kAcc], 0, nullptr, 0, nullptr);
    tmem_dealloc(tmem, L::kTmemCols);
  }
}

}  // namespace qtc

static int qtc_sms(int dev) {
  static int n[64] = {0};
  if (n[dev] == 0) cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev);
  return n[dev];
}

bool qass_tc_supported(int64_t H, int64_t D) {
  const char* env = std::getenv("NORI_QASS_TC");
  if (env != nullptr && env[0] == '0') return false;
  return H >= 1 && H <= qtc::kMaxHeads && 128 % H == 0 && D >= 8 && D <= 64 && D % 8 == 0;
}

// Launch the tensor-core QASS kernel. `dout`/`gs`/`gw*`/`gb*` are used by the backward only.
void qass_tc_launch(bool bwd, const torch::Tensor& q, const torch::Tensor* dout, torch::Tensor& out,
                    const float* s, const float* w1, const float* b1, const float* w2, const float* b2, float* gs,
                    float* gw1, float* gb1, float* gw2, float* gb2, int64_t H, int64_t D, int* status) {
  const int64_t R = q.size(0);
  const int dev = q.get_device();
  int64_t qdims[3] = {D, H, R};
  int64_t qstr[2] = {D * 2, q.stride(0) * 2};
  int qbox[3] = {64, static_cast<int>(H), static_cast<int>(128 / H)};
  CUtensorMap tmq = make_tmap_nd_bf16(q.data_ptr(), 3, qdims, qstr, qbox);
  CUtensorMap tmdo = tmq;
  if (bwd) {
    int64_t ddims[3] = {D, H, R};
    int64_t dstr[2] = {D * 4, dout->stride(0) * 4};
    int dbox[3] = {32, static_cast<int>(H), static_cast<int>(128 / H)};
    tmdo = make_tmap_nd_bf16(dout->data_ptr(), 3, ddims, dstr, dbox, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_DATA_TYPE_FLOAT32);
  }
  qtc::Params p{};
  p.nvec = R * H;
  p.H = static_cast<int>(H);
  p.D = static_cast<int>(D);
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ldo = out.stride(0);
  p.w1 = w1;
  p.b1 = b1;
  p.w2 = w2;
  p.b2 = b2;
  p.s = s;
  p.gw1 = gw1;
  p.gb1 = gb1;
  p.gw2 = gw2;
  p.gb2 = gb2;
  p.gs = gs;
  p.status = status;
  const int64_t tiles = (p.nvec + 127) / 128;
  auto stream = at::cuda::getCurrentCUDAStream();
  static int set_f[64] = {0}, set_b[64] = {0};
  if (bwd) {
    constexpr int smem = qtc::Lay<true>::kAlloc;
    if (!set_b[dev]) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(qtc::qass_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      set_b[dev] = 1;
    }
    const int grid = static_cast<int>(std::min<int64_t>(tiles, persistent_sms(qtc_sms(dev))));
    qtc::qass_tc_kernel<true><<<grid, qtc::kThreads, smem, stream>>>(tmq, tmdo, p);
  } else {
    constexpr int smem = qtc::Lay<false>::kAlloc;
    if (!set_f[dev]) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(qtc::qass_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      set_f[dev] = 1;
    }
    const int grid = static_cast<int>(std::min<int64_t>(tiles, persistent_sms(qtc_sms(dev))));
    qtc::qass_tc_kernel<false><<<grid, qtc::kThreads, smem, stream>>>(tmq, tmdo, p);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace nori
