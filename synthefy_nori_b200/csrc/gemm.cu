// Persistent tcgen05 GEMM for sm_100a with fused epilogues.
//
//   C[M, N] = A[M, K] . B[N, K]^T     (bf16 operands, fp32 accumulation in TMEM)
//
// Operands may be K-major (row-major [rows, K]) or MN-major (the transpose stored
// row-major, i.e. [K, rows]); the forward projections use K-major x K-major, the
// input-gradient GEMM K-major x MN-major (dX = dY W, no transposed weight copy) and
// the weight-gradient GEMM MN-major x MN-major with split-K over tokens
// (dW = dY^T X accumulated in fp32).
//
// One CTA per SM walks work items (128 x BN output tile, K range). Warp roles
// (320 threads):
//   warp 0      TMA producer: 128B-swizzled boxes into an S-stage ring (full/empty
//               mbarriers); no cluster multicast;
//   warp 1      TMEM owner + MMA issuer: one elected thread issues tcgen05.mma
//               (M=128, N=BN, K=16) into one of two TMEM accumulators so the epilogue
//               of item i overlaps the main loop of item i+1;
//   warps 2..9  epilogue: two warps per TMEM lane quarter split the columns; 32-column
//               tcgen05.ld, the fused op, 64-byte-swizzled shared staging, and TMA bulk
//               stores of 128 x 32 boxes (tails clipped by the tensor map).
//
// Epilogues (ops the Nori encoder layer fuses into its GEMMs):
//   kStore    out = bf16(act(acc * row_scale[m] + bias[n]))   (RMSNorm without affine
//             weight commutes with the GEMM: rms(x) W^T = diag(r) x W^T; act = identity or
//             the exact GELU of a GELU MLP's first projection)
//   kSwiGLU   weight rows interleaved (gate_j, up_j): out[m, j] = silu(g r) * (u r)
//   kResidual out = bf16(resid[m, n] + alpha * acc) (resid tile TMA-loaded into the
//             staging buffer), with each row's sum of squares added to sumsq[m]
//   kF32Atomic out_f32[m, n] += acc (fp32 reduction, split-K weight gradients)
//   kSwiGLUBwd the SwiGLU pre-activation recomputed (gate / up rows interleaved, row scale)
//             and turned into its gradient in place: with dh[m, j] TMA-loaded beside the
//             staging buffer, out[m, 2j] = dh silu'(g) u, out[m, 2j + 1] = dh silu(g); the
//             pre-activation itself is never written
//
// Reference ops fused here: model/layer.py:233-258 (RMSNorm), 261-274 (SwiGLU),
// 1093-1162 (QKV / output projections), 1443-1446 (DeepNorm residual).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <atomic>

#include "sm100.cuh"
#include "tma_host.h"

namespace nori {

enum Epilogue : int { kStore = 0, kSwiGLU = 1, kResidual = 2, kF32Atomic = 3, kSwiGLUBwd = 4 };

struct GemmParams {
  int M, N, K;
  int k_blocks_per_split, k_splits;
  float* out_f32;
  int64_t ldo;
  const float* row_scale;  // [M] or null
  const float* bias;       // [N] or null
  float alpha;
  float* sumsq;  // [M] or null
  int act;       // kStore: 0 none, 1 exact GELU applied after scale and bias
  int* status;
};

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kGemmThreads = 320;
constexpr int kEpiThreads = 256;
constexpr int kBoxCols = 32;                 // staging / store box width (64 bytes of bf16)
constexpr int kBoxBytes = kBM * kBoxCols * 2;  // 8 KB

template <int BN, int EPI>
struct GemmCfg {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kOutCols = (EPI == kSwiGLU) ? BN / 2 : BN;
  static constexpr int kAuxBytes = (EPI == kSwiGLUBwd) ? kBM * (BN / 2) * 2 : 0;  // the dh tile
  static constexpr int kStagingBytes = (EPI == kF32Atomic) ? 0 : kBM * kOutCols * 2 + kAuxBytes;
  static constexpr int kBudget = 220 * 1024 - kStagingBytes;
  static constexpr int kStages = (kBudget / kStageBytes) > 8 ? 8 : (kBudget / kStageBytes);
  static constexpr int kTmemCols = (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
  static constexpr int kSmemBytes = kStages * kStageBytes + kStagingBytes + 1024 + 256;
  static_assert(kStages >= 2, "not enough shared memory for a 2-stage pipeline");
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "BN must be a multiple of 32 in [64, 256]");
};

// silu(x) = x sigmoid(x) = 0.5 x (1 + tanh(x / 2)): one MUFU instruction (tanh.approx, max
// relative error about 2^-11, below the bf16 output's 2^-9) instead of an exponential and a
// reciprocal; with 128 x BN outputs per tile the SwiGLU epilogue was bound by the MUFU.
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float silu_f(float x) {
  const float h = 0.5f * x;
  return fmaf(h, tanh_approx(h), h);
}

// byte offset of (row, 16-byte chunk c in 0..3) inside a 128 x 32 bf16 box with 64B swizzle
__device__ __forceinline__ int box_off(int row, int c) { return row * 64 + ((c ^ ((row >> 1) & 3)) << 4); }

template <int BN, int EPI, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmR, GemmParams p) {
  using Cfg = GemmCfg<BN, EPI>;
  constexpr int S = Cfg::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* staging = smem + S * Cfg::kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(staging + Cfg::kStagingBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* rbar = tempty + 2;
  uint64_t* ebar = rbar + 1;  // [2] bounded epilogue-group barriers (staging free / staging written)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ebar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int num_m = (p.M + kBM - 1) / kBM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_kb = (p.K + kBK - 1) / kBK;
  const int items = num_m * num_n * p.k_splits;
  // a CTA that starts after another one timed out returns at once
  if (p.status != nullptr && *reinterpret_cast<volatile int*>(p.status) != 0) return;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], kEpiThreads / 32);
    }
    mbar_init(rbar, 1);
    mbar_init(&ebar[0], kEpiThreads / 32);
    mbar_init(&ebar[1], kEpiThreads / 32);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cfg::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // item -> (mb, nb, ks); N-tiles of one M block are adjacent so the A block stays in L2
  auto decode = [&](int t, int& mb, int& nb, int& ks) {
    ks = t % p.k_splits;
    const int mn = t / p.k_splits;
    mb = mn / num_n;
    nb = mn % num_n;
  };
  auto k_range = [&](int ks, int& kb0, int& kb1) {
    kb0 = ks * p.k_blocks_per_split;
    kb1 = min(num_kb, kb0 + p.k_blocks_per_split);
  };

  if (warp == 0) {
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < items; t += gridDim.x) {
        int mb, nb, ks, kb0, kb1;
        decode(t, mb, nb, ks);
        k_range(ks, kb0, kb1);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.status, kTimeoutProducer, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * Cfg::kStageBytes;
          uint8_t* sb = sa + Cfg::kABytes;
          mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
          if constexpr (A_MN) {
            tma_load_2d(sa, &tmA, &full[stage], mb * kBM, kb * kBK);
            tma_load_2d(sa + 8192, &tmA, &full[stage], mb * kBM + 64, kb * kBK);
          } else {
            tma_load_2d(sa, &tmA, &full[stage], kb * kBK, mb * kBM);
          }
          if constexpr (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(sb + j * 8192, &tmB, &full[stage], nb * BN + j * 64, kb * kBK);
          } else {
            tma_load_2d(sb, &tmB, &full[stage], kb * kBK, nb * BN);
          }
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = umma_idesc_bf16(kBM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int t = blockIdx.x; t < items; t += gridDim.x) {
        int mb, nb, ks, kb0, kb1;
        decode(t, mb, nb, ks);
        k_range(ks, kb0, kb1);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, p.status, kTimeoutMma, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.status, kTimeoutMma, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * Cfg::kStageBytes);
          const uint32_t sb = sa + Cfg::kABytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            uint64_t da, db;
            if constexpr (A_MN) {
              da = umma_smem_desc(sa + k * 2048, 8192, 1024, 2);
            } else {
              da = umma_desc_kmajor_sw128(sa + k * 32);
            }
            if constexpr (B_MN) {
              db = umma_smem_desc(sb + k * 2048, 8192, 1024, 2);
            } else {
              db = umma_desc_kmajor_sw128(sb + k * 32);
            }
            umma_bf16_ss(d_tmem, da, db, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int e_tid = threadIdx.x - 64;
    const int q = warp & 3;          // TMEM lane quarter
    const int half = (warp - 2) >> 2;  // column half (32-column chunks alternate)
    const int r_in = q * 32 + lane;  // row inside the tile
    int acc = 0;
    uint32_t acc_phase = 0, r_phase = 0, e_phase = 0;
    for (int t = blockIdx.x; t < items; t += gridDim.x) {
      int mb, nb, ks;
      decode(t, mb, nb, ks);
      const int m0 = mb * kBM, n0 = nb * BN;
      if constexpr (EPI != kF32Atomic) {
        if (e_tid == 0) {
          bulk_wait_read0();
          if constexpr (EPI == kResidual) {
            mbar_arrive_expect_tx(rbar, Cfg::kStagingBytes);
#pragma unroll
            for (int j = 0; j < BN / kBoxCols; ++j) tma_load_2d(staging + j * kBoxBytes, &tmR, rbar, n0 + j * kBoxCols, m0);
          }
          if constexpr (EPI == kSwiGLUBwd) {
            mbar_arrive_expect_tx(rbar, Cfg::kAuxBytes);
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(staging + kBM * BN * 2 + j * kBoxBytes, &tmR, rbar, n0 / 2 + j * kBoxCols, m0);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&ebar[0]);
        if (!mbar_wait_warp(&ebar[0], e_phase, p.status, kTimeoutEpilogue, abort_flag)) break;
      }
      if (!mbar_wait_warp(&tfull[acc], acc_phase, p.status, kTimeoutEpilogue, abort_flag)) break;
      if constexpr (EPI == kResidual || EPI == kSwiGLUBwd) {
        if (!mbar_wait_warp(rbar, r_phase, p.status, kTimeoutEpilogue, abort_flag)) break;
        r_phase ^= 1;
      }
      tc_fence_after();
      const int row = m0 + r_in;
      const bool row_ok = row < p.M;
      const float rs = (p.row_scale != nullptr && row_ok) ? p.row_scale[row] : 1.0f;
      float ssq = 0.f;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = half; c < BN / 32; c += 2) {
        uint32_t r[32];
        tmem_ld32(taddr + c * 32, r);
        tmem_wait_ld();
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
        if constexpr (EPI == kStore) {
          uint8_t* box = staging + c * kBoxBytes;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            v[i] *= rs * p.alpha;
            if (p.bias != nullptr) {
              const int col = n0 + c * 32 + i;
              if (col < p.N) v[i] += p.bias[col];
            }
          }
          if (p.act == 1) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = 0.5f * v[i] * (1.0f + erff(v[i] * 0.70710678118654752f));
          }
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            uint4 w = make_uint4(pack_bf16x2(v[8 * cc], v[8 * cc + 1]), pack_bf16x2(v[8 * cc + 2], v[8 * cc + 3]),
                                 pack_bf16x2(v[8 * cc + 4], v[8 * cc + 5]), pack_bf16x2(v[8 * cc + 6], v[8 * cc + 7]));
            *reinterpret_cast<uint4*>(box + box_off(r_in, cc)) = w;
          }
        } else if constexpr (EPI == kSwiGLU) {
          // 32 accumulator columns -> 16 output columns = half of output box c / 2
          uint8_t* box = staging + (c >> 1) * kBoxBytes;
          float h[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) h[i] = silu_f(v[2 * i] * rs) * (v[2 * i + 1] * rs);
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            uint4 w = make_uint4(pack_bf16x2(h[8 * cc], h[8 * cc + 1]), pack_bf16x2(h[8 * cc + 2], h[8 * cc + 3]),
                                 pack_bf16x2(h[8 * cc + 4], h[8 * cc + 5]), pack_bf16x2(h[8 * cc + 6], h[8 * cc + 7]));
            *reinterpret_cast<uint4*>(box + box_off(r_in, (c & 1) * 2 + cc)) = w;
          }
        } else if constexpr (EPI == kResidual) {
          uint8_t* box = staging + c * kBoxBytes;
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            uint4* slot = reinterpret_cast<uint4*>(box + box_off(r_in, cc));
            const uint4 rv = *slot;
            const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
            uint32_t pk[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float lo = bf16lo(rw[i]) + p.alpha * v[8 * cc + 2 * i];
              const float hi = bf16hi(rw[i]) + p.alpha * v[8 * cc + 2 * i + 1];
              pk[i] = pack_bf16x2(lo, hi);
              const int col = n0 + c * 32 + 8 * cc + 2 * i;
              const float blo = bf16lo(pk[i]), bhi = bf16hi(pk[i]);
              if (col < p.N) ssq += blo * blo;
              if (col + 1 < p.N) ssq += bhi * bhi;
            }
            *slot = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          }
        } else if constexpr (EPI == kSwiGLUBwd) {
          // 32 accumulator columns = 16 (gate, up) pairs, whose dh values are 16 columns of
          // the dh tile: half (c & 1) of dh box c / 2
          const uint8_t* dbox = staging + kBM * BN * 2 + (c >> 1) * kBoxBytes;
          float dh[16];
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            const uint4 w = *reinterpret_cast<const uint4*>(dbox + box_off(r_in, (c & 1) * 2 + cc));
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              dh[cc * 8 + 2 * i] = bf16lo(ww[i]);
              dh[cc * 8 + 2 * i + 1] = bf16hi(ww[i]);
            }
          }
          float o[32];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float g = v[2 * i] * rs, u = v[2 * i + 1] * rs;
            const float sig = fmaf(0.5f, tanh_approx(0.5f * g), 0.5f);  // sigmoid(g)
            const float dsilu = sig * fmaf(g, 1.0f - sig, 1.0f);         // silu'(g)
            o[2 * i] = dh[i] * u * dsilu;
            o[2 * i + 1] = dh[i] * (g * sig);
          }
          uint8_t* box = staging + c * kBoxBytes;
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            uint4 w = make_uint4(pack_bf16x2(o[8 * cc], o[8 * cc + 1]), pack_bf16x2(o[8 * cc + 2], o[8 * cc + 3]),
                                 pack_bf16x2(o[8 * cc + 4], o[8 * cc + 5]), pack_bf16x2(o[8 * cc + 6], o[8 * cc + 7]));
            *reinterpret_cast<uint4*>(box + box_off(r_in, cc)) = w;
          }
        } else if constexpr (EPI == kF32Atomic) {
          if (row_ok) {
            float* o = p.out_f32 + static_cast<int64_t>(row) * p.ldo + n0 + c * 32;
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (n0 + c * 32 + i < p.N) atomicAdd(o + i, p.alpha * v[i]);
          }
        }
      }
      if constexpr (EPI == kResidual) {
        if (p.sumsq != nullptr && row_ok) atomicAdd(&p.sumsq[row], ssq);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
      if constexpr (EPI != kF32Atomic) {
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ebar[1]);
        if (!mbar_wait_warp(&ebar[1], e_phase, p.status, kTimeoutEpilogue, abort_flag)) break;
        e_phase ^= 1;
        if (e_tid == 0) {
          const int n0_out = (EPI == kSwiGLU) ? n0 / 2 : n0;
#pragma unroll
          for (int j = 0; j < Cfg::kOutCols / kBoxCols; ++j)
            tma_store_2d(&tmC, staging + j * kBoxBytes, n0_out + j * kBoxCols, m0);
          bulk_commit();
        }
      }
    }
    if constexpr (EPI != kF32Atomic) {
      if (e_tid == 0) bulk_wait0();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// ------------------------------------------------------------------ host side
static std::atomic<int> g_sm_reserve{0};
int sm_reserve() { return g_sm_reserve.load(std::memory_order_relaxed); }
void set_sm_reserve(int64_t n) {
  TORCH_CHECK(n >= 0 && n < 64, "sm_reserve must be in [0, 64)");
  g_sm_reserve.store(static_cast<int>(n), std::memory_order_relaxed);
}

static int num_sms(int dev) {
  static int cache[64] = {0};
  if (cache[dev] == 0) cudaDeviceGetAttribute(&cache[dev], cudaDevAttrMultiProcessorCount, dev);
  return cache[dev];
}

struct Operand {
  const torch::Tensor* t;
  bool mn_major;  // tensor is [K, rows] (rows contiguous) instead of [rows, K]
};

static CUtensorMap operand_map(const Operand& o, int rows, int K, int box_rows) {
  const torch::Tensor& t = *o.t;
  if (o.mn_major) {
    // tensor [K, rows], rows contiguous; box = 64 rows (inner) x 64 K
    return make_tmap_2d_bf16(t.data_ptr(), rows, K, t.stride(0), 64, kBK);
  }
  return make_tmap_2d_bf16(t.data_ptr(), K, rows, t.stride(0), kBK, box_rows);
}

template <int BN, int EPI, bool A_MN, bool B_MN>
static void launch_gemm(const Operand& A, const Operand& B, const torch::Tensor* C, const torch::Tensor* R,
                        GemmParams& p, cudaStream_t stream) {
  using Cfg = GemmCfg<BN, EPI>;
  CUtensorMap ta = operand_map(A, p.M, p.K, kBM);
  CUtensorMap tb = operand_map(B, p.N, p.K, BN);
  CUtensorMap tc{}, tr{};
  if (C != nullptr)
    tc = make_tmap_2d_bf16(C->data_ptr(), C->size(1), C->size(0), C->stride(0), kBoxCols, kBM,
                           CU_TENSOR_MAP_SWIZZLE_64B);
  if (R != nullptr)
    tr = make_tmap_2d_bf16(R->data_ptr(), R->size(1), R->size(0), R->stride(0), kBoxCols, kBM,
                           CU_TENSOR_MAP_SWIZZLE_64B);
  auto kern = gemm_kernel<BN, EPI, A_MN, B_MN>;
  const int dev = A.t->get_device();
  static bool configured[64] = {false};
  if (!configured[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
    configured[dev] = true;
  }
  const int items = ((p.M + kBM - 1) / kBM) * ((p.N + BN - 1) / BN) * p.k_splits;
  const int grid = std::max(1, std::min(items, persistent_sms(num_sms(dev))));
  kern<<<grid, kGemmThreads, Cfg::kSmemBytes, stream>>>(ta, tb, tc, tr, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int EPI, bool A_MN, bool B_MN>
static void dispatch_bn(int bn, const Operand& A, const Operand& B, const torch::Tensor* C, const torch::Tensor* R,
                        GemmParams& p, cudaStream_t s) {
  switch (bn) {
    case 128: return launch_gemm<128, EPI, A_MN, B_MN>(A, B, C, R, p, s);
    case 192: return launch_gemm<192, EPI, A_MN, B_MN>(A, B, C, R, p, s);
    case 256: return launch_gemm<256, EPI, A_MN, B_MN>(A, B, C, R, p, s);
    default: TORCH_CHECK(false, "unsupported tile N ", bn);
  }
}

// Least padded columns plus a per-tile overhead; ties go to the wider tile.
static int choose_bn(int N, bool multiple_of_64_only = true) {
  (void)multiple_of_64_only;
  const int cands[] = {256, 192, 128};
  int best = 256;
  double best_cost = 1e30;
  for (int bn : cands) {
    const int tiles = (N + bn - 1) / bn;
    const double cost = static_cast<double>(tiles) * bn + tiles * 32.0;
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

static void check_operand(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 2, name, ": 2-D bf16 CUDA tensor expected");
  TORCH_CHECK(t.stride(1) == 1 && t.stride(0) % 8 == 0, name, ": row-major with 16-byte aligned rows expected");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name, ": 16-byte aligned base expected");
}

static GemmParams make_params(int M, int N, int K, const torch::Tensor& status) {
  GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.k_splits = 1;
  p.k_blocks_per_split = (K + kBK - 1) / kBK;
  p.alpha = 1.f;
  p.status = status.defined() && status.numel() > 0 ? status.data_ptr<int>() : nullptr;
  return p;
}

static const float* opt_f32(const c10::optional<torch::Tensor>& t, int64_t n, const char* what) {
  if (!t.has_value() || !t->defined()) return nullptr;
  TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() >= n, what,
              ": contiguous fp32 tensor of sufficient size expected");
  return t->data_ptr<float>();
}

// out = bf16(act((A @ W^T) * row_scale[:, None] + bias)).  A [M, K]; W [N, K] (or w_kn: W stored [K, N]).
torch::Tensor gemm_bf16(const torch::Tensor& A, const torch::Tensor& W, const c10::optional<torch::Tensor>& row_scale,
                        const c10::optional<torch::Tensor>& bias, const torch::Tensor& status, int64_t bn, bool w_kn,
                        double alpha, const c10::optional<torch::Tensor>& out_opt, int64_t act) {
  check_operand(A, "A");
  check_operand(W, "W");
  const int64_t N = w_kn ? W.size(1) : W.size(0);
  const int64_t K = w_kn ? W.size(0) : W.size(1);
  TORCH_CHECK(A.size(1) == K, "gemm: K mismatch");
  TORCH_CHECK(N % 8 == 0, "gemm: N must be a multiple of 8");
  const at::cuda::CUDAGuard guard(A.device());
  torch::Tensor out = out_opt.has_value() && out_opt->defined() ? *out_opt : torch::empty({A.size(0), N}, A.options());
  check_operand(out, "out");
  TORCH_CHECK(out.size(0) == A.size(0) && out.size(1) == N, "gemm: out must be [M, N]");
  if (A.size(0) == 0) return out;
  GemmParams p = make_params(static_cast<int>(A.size(0)), static_cast<int>(N), static_cast<int>(K), status);
  p.row_scale = opt_f32(row_scale, p.M, "row_scale");
  p.bias = opt_f32(bias, p.N, "bias");
  p.alpha = static_cast<float>(alpha);
  TORCH_CHECK(act == 0 || act == 1, "gemm: act must be 0 (none) or 1 (gelu)");
  p.act = static_cast<int>(act);
  const int b = bn > 0 ? static_cast<int>(bn) : choose_bn(p.N);
  Operand oa{&A, false}, ow{&W, w_kn};
  auto s = at::cuda::getCurrentCUDAStream();
  if (w_kn)
    dispatch_bn<kStore, false, true>(b, oa, ow, &out, nullptr, p, s);
  else
    dispatch_bn<kStore, false, false>(b, oa, ow, &out, nullptr, p, s);
  return out;
}

// out[:, j] = silu(g_j r) * (u_j r) with W rows interleaved (gate_0, up_0, gate_1, ...)
torch::Tensor gemm_swiglu(const torch::Tensor& A, const torch::Tensor& W, const c10::optional<torch::Tensor>& row_scale,
                          const torch::Tensor& status, int64_t bn) {
  check_operand(A, "A");
  check_operand(W, "W");
  TORCH_CHECK(A.size(1) == W.size(1), "gemm_swiglu: K mismatch");
  TORCH_CHECK(W.size(0) % 16 == 0, "gemm_swiglu: 2*hidden must be a multiple of 16");
  const at::cuda::CUDAGuard guard(A.device());
  auto out = torch::empty({A.size(0), W.size(0) / 2}, A.options());
  if (A.size(0) == 0) return out;
  GemmParams p = make_params(static_cast<int>(A.size(0)), static_cast<int>(W.size(0)), static_cast<int>(A.size(1)), status);
  p.row_scale = opt_f32(row_scale, p.M, "row_scale");
  Operand oa{&A, false}, ow{&W, false};
  dispatch_bn<kSwiGLU, false, false>(bn > 0 ? static_cast<int>(bn) : choose_bn(p.N), oa, ow, &out, nullptr, p,
                                     at::cuda::getCurrentCUDAStream());
  return out;
}

// Gradient of the SwiGLU pre-activation: W rows interleaved (gate_0, up_0, ...) as for
// gemm_swiglu, dh [M, N / 2] the gradient of h = silu(g) u; returns [M, N] interleaved
// (d gate, d up) with g, u recomputed as (A W^T) * row_scale. Default tile N 256 (measured
// 709 TFLOP/s at 131072 x 2688 x 448 against 694 for 192 and 636 for 128).
torch::Tensor gemm_swiglu_bwd(const torch::Tensor& A, const torch::Tensor& W, const c10::optional<torch::Tensor>& row_scale,
                              const torch::Tensor& dh, const torch::Tensor& status, int64_t bn) {
  check_operand(A, "A");
  check_operand(W, "W");
  check_operand(dh, "dh");
  TORCH_CHECK(A.size(1) == W.size(1), "gemm_swiglu_bwd: K mismatch");
  TORCH_CHECK(W.size(0) % 16 == 0, "gemm_swiglu_bwd: 2*hidden must be a multiple of 16");
  TORCH_CHECK(dh.size(0) == A.size(0) && dh.size(1) * 2 == W.size(0), "gemm_swiglu_bwd: dh must be [M, hidden]");
  const at::cuda::CUDAGuard guard(A.device());
  auto out = torch::empty({A.size(0), W.size(0)}, A.options());
  if (A.size(0) == 0) return out;
  GemmParams p = make_params(static_cast<int>(A.size(0)), static_cast<int>(W.size(0)), static_cast<int>(A.size(1)), status);
  p.row_scale = opt_f32(row_scale, p.M, "row_scale");
  Operand oa{&A, false}, ow{&W, false};
  dispatch_bn<kSwiGLUBwd, false, false>(bn > 0 ? static_cast<int>(bn) : 256, oa, ow, &out, &dh, p,
                                        at::cuda::getCurrentCUDAStream());
  return out;
}

// out = bf16(resid + alpha * (A @ W^T)); sumsq[m] += sum_n out[m, n]^2 (if given).
// W is [N, K], or with w_kn the same matrix stored [K, N] (an MN-major operand: the
// output projections read their [E_in, E_out] weights in place, no transposed copy).
torch::Tensor gemm_residual(const torch::Tensor& A, const torch::Tensor& W, const torch::Tensor& resid, double alpha,
                            const c10::optional<torch::Tensor>& sumsq, const torch::Tensor& status, int64_t bn,
                            const c10::optional<torch::Tensor>& out_opt, bool w_kn) {
  check_operand(A, "A");
  check_operand(W, "W");
  check_operand(resid, "resid");
  const int64_t N = w_kn ? W.size(1) : W.size(0);
  const int64_t K = w_kn ? W.size(0) : W.size(1);
  TORCH_CHECK(A.size(1) == K, "gemm_residual: K mismatch");
  TORCH_CHECK(resid.size(0) == A.size(0) && resid.size(1) == N, "gemm_residual: resid must be [M, N]");
  const at::cuda::CUDAGuard guard(A.device());
  torch::Tensor out =
      out_opt.has_value() && out_opt->defined() ? *out_opt : torch::empty({A.size(0), N}, A.options());
  check_operand(out, "out");
  TORCH_CHECK(out.size(0) == A.size(0) && out.size(1) == N, "gemm_residual: out must be [M, N]");
  if (A.size(0) == 0) return out;
  GemmParams p = make_params(static_cast<int>(A.size(0)), static_cast<int>(N), static_cast<int>(K), status);
  TORCH_CHECK(p.N % 8 == 0, "gemm_residual: N must be a multiple of 8");
  p.alpha = static_cast<float>(alpha);
  p.sumsq = const_cast<float*>(opt_f32(sumsq, p.M, "sumsq"));
  Operand oa{&A, false}, ow{&W, w_kn};
  const int b = bn > 0 ? static_cast<int>(bn) : choose_bn(p.N);
  auto s = at::cuda::getCurrentCUDAStream();
  if (w_kn)
    dispatch_bn<kResidual, false, true>(b, oa, ow, &out, &resid, p, s);
  else
    dispatch_bn<kResidual, false, false>(b, oa, ow, &out, &resid, p, s);
  return out;
}

// Weight gradient: out (fp32 [N_out, K_in]) += dY^T X, with dY [T, N_out], X [T, K_in]
// (both token-major, i.e. MN-major operands), split over tokens.
void gemm_wgrad(const torch::Tensor& dY, const torch::Tensor& X, torch::Tensor& out, const torch::Tensor& status,
                int64_t bn, int64_t splits, double alpha) {
  check_operand(dY, "dY");
  check_operand(X, "X");
  TORCH_CHECK(dY.size(0) == X.size(0), "gemm_wgrad: token count mismatch");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous() && out.size(0) == dY.size(1) &&
                  out.size(1) == X.size(1),
              "gemm_wgrad: contiguous fp32 [N_out, K_in] accumulator expected");
  const at::cuda::CUDAGuard guard(dY.device());
  const int T = static_cast<int>(dY.size(0));
  if (T == 0) return;
  GemmParams p = make_params(static_cast<int>(dY.size(1)), static_cast<int>(X.size(1)), T, status);
  p.out_f32 = out.data_ptr<float>();
  p.ldo = out.stride(0);
  p.alpha = static_cast<float>(alpha);
  const int b = bn > 0 ? static_cast<int>(bn) : choose_bn(p.N);
  const int tiles = ((p.M + kBM - 1) / kBM) * ((p.N + b - 1) / b);
  const int num_kb = (T + kBK - 1) / kBK;
  int sp = splits > 0 ? static_cast<int>(splits) : std::max(1, (2 * num_sms(dY.get_device()) + tiles - 1) / tiles);
  sp = std::min(sp, num_kb);
  p.k_blocks_per_split = (num_kb + sp - 1) / sp;
  p.k_splits = (num_kb + p.k_blocks_per_split - 1) / p.k_blocks_per_split;
  Operand oa{&dY, true}, ox{&X, true};
  dispatch_bn<kF32Atomic, true, true>(b, oa, ox, nullptr, nullptr, p, at::cuda::getCurrentCUDAStream());
}

}  // namespace nori
