// Persistent tcgen05 GEMM for sm_100a with fused epilogues.
//
//   C[M, N] = A[M, K] . B[N, K]^T     (A, B bf16, K-major; fp32 accumulation in TMEM)
//
// One CTA per SM walks output tiles of 128 x BN. Warp roles (192 threads):
//   warp 0      TMA producer: 128B-swizzled A / B boxes of 64 K-elements into an
//               S-stage shared-memory ring (full / empty mbarriers);
//   warp 1      TMEM owner + MMA issuer: one elected thread issues tcgen05.mma
//               (M=128, N=BN, K=16) into one of two TMEM accumulators, so the
//               epilogue of tile i overlaps the main loop of tile i+1;
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (one output row per
//               thread), the fused operation, and the global store.
//
// Epilogues (the ops that the Nori encoder layer fuses into its GEMMs):
//   kStore    out = bf16(acc * row_scale[m] + bias[n])           (row_scale: RMSNorm
//             without affine weight commutes with the GEMM: rms(x) W = diag(r) x W)
//   kSwiGLU   weight rows interleaved (gate_j, up_j): out[m, j] = silu(g r) * (u r)
//   kResidual out = bf16(resid[m, n] + alpha * acc), and sum of squares of the new
//             row accumulated into sumsq[m] for the next RMSNorm
//   kF32      out_f32 = acc (optionally accumulated: out += acc)
//   kHeadMajor bf16(acc * row_scale) scattered into [blocks, T, 3?, H, N, Dp] layouts
//             used by the attention kernels (see HeadMajorMap).
//
// Reference ops fused here: model/layer.py:233-258 (RMSNorm), 261-274 (SwiGLU),
// 1093-1162 (QKV / out projections), 1443-1446 (DeepNorm residual).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <mutex>

#include "sm100.cuh"
#include "tma_host.h"

namespace nori {

enum Epilogue : int { kStore = 0, kSwiGLU = 1, kResidual = 2, kF32 = 3, kHeadMajor = 4 };

// Destination map of the head-major scatter: row m = (blk, n, t) with
// blk = m / (n_rows * T), n = (m / T) % n_rows, t = m % T; column c = (j, h, d) with
// j = c / (H * D), h = (c / D) % H, d = c % D. Element goes to
//   out[(((blk * T + t) * J + j) * H + h) * n_rows + n) * Dp + d]
// i.e. per (blk, t, j, h) a contiguous [n_rows, Dp] matrix (Dp >= D, zero padded by the
// caller's allocation being pre-zeroed once; padding columns are never written).
struct HeadMajorMap {
  int T, n_rows, J, H, D, Dp;
};

struct GemmParams {
  int M, N, K;
  void* out;
  int64_t ldo;
  const float* row_scale;  // [M] or null
  const float* bias;       // [N] or null
  const __nv_bfloat16* resid;
  int64_t ldr;
  float alpha;
  float* sumsq;  // [M] or null
  int accumulate;
  HeadMajorMap hm;
  int* status;
};

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 192;

template <int BN>
struct GemmCfg {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (200 * 1024) / kStageBytes > 8 ? 8 : (200 * 1024) / kStageBytes;
  static constexpr int kTmemCols = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmParams p) {
  using Cfg = GemmCfg<BN>;
  constexpr int S = Cfg::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int num_m = (p.M + kBM - 1) / kBM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_k = (p.K + kBK - 1) / kBK;
  const int tiles = num_m * num_n;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
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

  if (warp == 0) {
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
        const int mb = t / num_n, nb = t % num_n;
        bool ok = true;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.status, kTimeoutProducer, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * Cfg::kStageBytes;
          uint8_t* sb = sa + Cfg::kABytes;
          mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
          tma_load_2d(sa, &tmA, &full[stage], kb * kBK, mb * kBM);
          tma_load_2d(sb, &tmB, &full[stage], kb * kBK, nb * BN);
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
      constexpr uint32_t idesc = umma_idesc_bf16(kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, p.status, kTimeoutMma, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.status, kTimeoutMma, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * Cfg::kStageBytes);
          const uint32_t sb = sa + Cfg::kABytes;
          const uint64_t da = umma_desc_kmajor_sw128(sa);
          const uint64_t db = umma_desc_kmajor_sw128(sb);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            // advance the start address by k * 32 bytes inside the swizzle atom
            umma_bf16_ss(d_tmem, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
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
    // epilogue warps 2..5 -> TMEM lane quarter (warp % 4)
    const int q = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      const int mb = t / num_n, nb = t % num_n;
      if (!mbar_wait(&tfull[acc], acc_phase, p.status, kTimeoutEpilogue, abort_flag)) break;
      tc_fence_after();
      const int row = mb * kBM + q * 32 + lane;
      const bool row_ok = row < p.M;
      const float rs = (p.row_scale != nullptr && row_ok) ? p.row_scale[row] : 1.0f;
      float ssq = 0.f;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        uint32_t r[16];
        tmem_ld16(taddr + c, r);
        tmem_wait_ld();
        const int n0 = nb * BN + c;
        if (!row_ok || n0 >= p.N) continue;
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
        const bool full16 = (n0 + 16 <= p.N);
        if constexpr (EPI == kStore) {
          __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<int64_t>(row) * p.ldo + n0;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            v[i] *= rs;
            if (p.bias != nullptr && n0 + i < p.N) v[i] += p.bias[n0 + i];
          }
          if (full16) {
            uint4 w0 = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                                  pack_bf16x2(v[6], v[7]));
            uint4 w1 = make_uint4(pack_bf16x2(v[8], v[9]), pack_bf16x2(v[10], v[11]), pack_bf16x2(v[12], v[13]),
                                  pack_bf16x2(v[14], v[15]));
            reinterpret_cast<uint4*>(o)[0] = w0;
            reinterpret_cast<uint4*>(o)[1] = w1;
          } else {
            for (int i = 0; i < 16 && n0 + i < p.N; ++i) o[i] = __float2bfloat16(v[i]);
          }
        } else if constexpr (EPI == kSwiGLU) {
          // N counts interleaved (gate, up) columns; output has N / 2 columns.
          __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<int64_t>(row) * p.ldo + n0 / 2;
          float h[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) h[i] = silu_f(v[2 * i] * rs) * (v[2 * i + 1] * rs);
          if (full16) {
            *reinterpret_cast<uint4*>(o) = make_uint4(pack_bf16x2(h[0], h[1]), pack_bf16x2(h[2], h[3]),
                                                      pack_bf16x2(h[4], h[5]), pack_bf16x2(h[6], h[7]));
          } else {
            for (int i = 0; i < 8 && n0 + 2 * i < p.N; ++i) o[i] = __float2bfloat16(h[i]);
          }
        } else if constexpr (EPI == kResidual) {
          __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<int64_t>(row) * p.ldo + n0;
          const __nv_bfloat16* rr = p.resid + static_cast<int64_t>(row) * p.ldr + n0;
          if (full16) {
            uint4 a0 = reinterpret_cast<const uint4*>(rr)[0];
            uint4 a1 = reinterpret_cast<const uint4*>(rr)[1];
            uint32_t rw[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              v[2 * i] = bf16lo(rw[i]) + p.alpha * v[2 * i];
              v[2 * i + 1] = bf16hi(rw[i]) + p.alpha * v[2 * i + 1];
            }
            uint32_t pk[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              pk[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
              const float lo = bf16lo(pk[i]), hi = bf16hi(pk[i]);
              ssq += lo * lo + hi * hi;
            }
            reinterpret_cast<uint4*>(o)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            reinterpret_cast<uint4*>(o)[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
          } else {
            for (int i = 0; i < 16 && n0 + i < p.N; ++i) {
              const float x = __bfloat162float(rr[i]) + p.alpha * v[i];
              const __nv_bfloat16 b = __float2bfloat16(x);
              const float xb = __bfloat162float(b);
              ssq += xb * xb;
              o[i] = b;
            }
          }
        } else if constexpr (EPI == kF32) {
          float* o = reinterpret_cast<float*>(p.out) + static_cast<int64_t>(row) * p.ldo + n0;
          for (int i = 0; i < 16 && n0 + i < p.N; ++i) o[i] = p.accumulate ? o[i] + v[i] : v[i];
        } else if constexpr (EPI == kHeadMajor) {
          const HeadMajorMap& hm = p.hm;
          const int rows_per_blk = hm.n_rows * hm.T;
          const int blk = row / rows_per_blk;
          const int rem = row - blk * rows_per_blk;
          const int n = rem / hm.T;
          const int tt = rem - n * hm.T;
          __nv_bfloat16* base = reinterpret_cast<__nv_bfloat16*>(p.out);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int col = n0 + i;
            if (col >= p.N) break;
            const int d = col % hm.D;
            const int hh = (col / hm.D) % hm.H;
            const int j = col / (hm.D * hm.H);
            const int64_t idx =
                ((((static_cast<int64_t>(blk) * hm.T + tt) * hm.J + j) * hm.H + hh) * hm.n_rows + n) * hm.Dp + d;
            base[idx] = __float2bfloat16(v[i] * rs);
          }
        }
      }
      if constexpr (EPI == kResidual) {
        if (p.sumsq != nullptr && row_ok) atomicAdd(&p.sumsq[row], ssq);
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
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
static int num_sms(int dev) {
  static int cache[64] = {0};
  if (cache[dev] == 0) cudaDeviceGetAttribute(&cache[dev], cudaDevAttrMultiProcessorCount, dev);
  return cache[dev];
}

template <int BN, int EPI>
static void launch_gemm(const torch::Tensor& A, const torch::Tensor& B, GemmParams& p, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  CUtensorMap ta = make_tmap_2d_bf16(A.data_ptr(), p.K, p.M, A.stride(0), kBK, kBM);
  CUtensorMap tb = make_tmap_2d_bf16(B.data_ptr(), p.K, B.size(0), B.stride(0), kBK, BN);
  auto kern = gemm_tn_kernel<BN, EPI>;
  static bool configured[64] = {false};
  const int dev = A.get_device();
  if (!configured[dev]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    configured[dev] = true;
  }
  const int tiles = ((p.M + kBM - 1) / kBM) * ((p.N + BN - 1) / BN);
  const int grid = std::max(1, std::min(tiles, num_sms(dev)));
  kern<<<grid, kThreads, Cfg::kSmemBytes, stream>>>(ta, tb, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int EPI>
static void dispatch_bn(int bn, const torch::Tensor& A, const torch::Tensor& B, GemmParams& p, cudaStream_t s) {
  switch (bn) {
    case 64: return launch_gemm<64, EPI>(A, B, p, s);
    case 128: return launch_gemm<128, EPI>(A, B, p, s);
    case 192: return launch_gemm<192, EPI>(A, B, p, s);
    case 224: return launch_gemm<224, EPI>(A, B, p, s);
    case 256: return launch_gemm<256, EPI>(A, B, p, s);
    default: TORCH_CHECK(false, "unsupported tile N ", bn);
  }
}

// Pick the tile width with the least padding waste (ties -> wider tile).
static int choose_bn(int N) {
  const int cands[] = {256, 224, 192, 128, 64};
  int best = 256;
  double best_cost = 1e30;
  for (int bn : cands) {
    const int tiles = (N + bn - 1) / bn;
    // cost: padded columns plus a fixed per-tile overhead (epilogue / pipeline fill)
    const double cost = static_cast<double>(tiles) * bn + tiles * 24.0;
    if (cost < best_cost) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

static void check_operands(const torch::Tensor& A, const torch::Tensor& B) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda(), "gemm: CUDA tensors expected");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm: bf16 operands expected");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2, "gemm: 2-D operands expected");
  TORCH_CHECK(A.size(1) == B.size(1), "gemm: K mismatch");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1, "gemm: K-major (row-major) operands expected");
  TORCH_CHECK(A.stride(0) % 8 == 0 && B.stride(0) % 8 == 0, "gemm: row strides must be multiples of 16 bytes");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(A.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(B.data_ptr()) % 16 == 0,
              "gemm: operands must be 16-byte aligned");
}

static GemmParams base_params(const torch::Tensor& A, const torch::Tensor& B, const torch::Tensor& status) {
  GemmParams p{};
  p.M = static_cast<int>(A.size(0));
  p.N = static_cast<int>(B.size(0));
  p.K = static_cast<int>(A.size(1));
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

// out = bf16((A @ B^T) * row_scale[:, None] + bias)
torch::Tensor gemm_bf16(const torch::Tensor& A, const torch::Tensor& B, const c10::optional<torch::Tensor>& row_scale,
                        const c10::optional<torch::Tensor>& bias, const torch::Tensor& status, int64_t bn) {
  check_operands(A, B);
  const at::cuda::CUDAGuard guard(A.device());
  auto out = torch::empty({A.size(0), B.size(0)}, A.options());
  GemmParams p = base_params(A, B, status);
  if (p.M == 0 || p.N == 0) return out;
  p.out = out.data_ptr();
  p.ldo = out.stride(0);
  p.row_scale = opt_f32(row_scale, p.M, "row_scale");
  p.bias = opt_f32(bias, p.N, "bias");
  TORCH_CHECK(p.N % 8 == 0, "gemm_bf16: N must be a multiple of 8");
  dispatch_bn<kStore>(bn > 0 ? static_cast<int>(bn) : choose_bn(p.N), A, B, p, at::cuda::getCurrentCUDAStream());
  return out;
}

// out[:, j] = silu(g_j r) * (u_j r) with B rows interleaved (gate_0, up_0, gate_1, ...)
torch::Tensor gemm_swiglu(const torch::Tensor& A, const torch::Tensor& B, const c10::optional<torch::Tensor>& row_scale,
                          const torch::Tensor& status, int64_t bn) {
  check_operands(A, B);
  const at::cuda::CUDAGuard guard(A.device());
  TORCH_CHECK(B.size(0) % 16 == 0, "gemm_swiglu: 2*hidden must be a multiple of 16");
  auto out = torch::empty({A.size(0), B.size(0) / 2}, A.options());
  GemmParams p = base_params(A, B, status);
  if (p.M == 0) return out;
  p.out = out.data_ptr();
  p.ldo = out.stride(0);
  p.row_scale = opt_f32(row_scale, p.M, "row_scale");
  dispatch_bn<kSwiGLU>(bn > 0 ? static_cast<int>(bn) : choose_bn(p.N), A, B, p, at::cuda::getCurrentCUDAStream());
  return out;
}

// out = bf16(resid + alpha * (A @ B^T)); sumsq[m] += sum_n out[m, n]^2 (if given)
torch::Tensor gemm_residual(const torch::Tensor& A, const torch::Tensor& B, const torch::Tensor& resid, double alpha,
                            const c10::optional<torch::Tensor>& sumsq, const torch::Tensor& status, int64_t bn) {
  check_operands(A, B);
  const at::cuda::CUDAGuard guard(A.device());
  TORCH_CHECK(resid.scalar_type() == at::kBFloat16 && resid.dim() == 2 && resid.size(0) == A.size(0) &&
                  resid.size(1) == B.size(0) && resid.stride(1) == 1 && resid.stride(0) % 8 == 0,
              "gemm_residual: bf16 [M, N] residual with 16-byte rows expected");
  auto out = torch::empty({A.size(0), B.size(0)}, A.options());
  GemmParams p = base_params(A, B, status);
  if (p.M == 0) return out;
  TORCH_CHECK(p.N % 8 == 0, "gemm_residual: N must be a multiple of 8");
  p.out = out.data_ptr();
  p.ldo = out.stride(0);
  p.resid = reinterpret_cast<const __nv_bfloat16*>(resid.data_ptr());
  p.ldr = resid.stride(0);
  p.alpha = static_cast<float>(alpha);
  p.sumsq = const_cast<float*>(opt_f32(sumsq, p.M, "sumsq"));
  dispatch_bn<kResidual>(bn > 0 ? static_cast<int>(bn) : choose_bn(p.N), A, B, p, at::cuda::getCurrentCUDAStream());
  return out;
}

// out (fp32, [M, N]) = A @ B^T  (or += when accumulate)
void gemm_f32_out(const torch::Tensor& A, const torch::Tensor& B, torch::Tensor& out, bool accumulate,
                  const torch::Tensor& status, int64_t bn) {
  check_operands(A, B);
  const at::cuda::CUDAGuard guard(A.device());
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.dim() == 2 && out.size(0) == A.size(0) &&
                  out.size(1) == B.size(0) && out.stride(1) == 1,
              "gemm_f32_out: fp32 [M, N] output expected");
  GemmParams p = base_params(A, B, status);
  if (p.M == 0) return;
  p.out = out.data_ptr();
  p.ldo = out.stride(0);
  p.accumulate = accumulate ? 1 : 0;
  dispatch_bn<kF32>(bn > 0 ? static_cast<int>(bn) : choose_bn(p.N), A, B, p, at::cuda::getCurrentCUDAStream());
}

// Head-major projection: out[(blk, t, j, h), n, :Dp] = bf16((A @ B^T) * row_scale) (see HeadMajorMap).
void gemm_headmajor(const torch::Tensor& A, const torch::Tensor& B, const c10::optional<torch::Tensor>& row_scale,
                    torch::Tensor& out, int64_t T, int64_t n_rows, int64_t J, int64_t H, int64_t D, int64_t Dp,
                    const torch::Tensor& status, int64_t bn) {
  check_operands(A, B);
  const at::cuda::CUDAGuard guard(A.device());
  GemmParams p = base_params(A, B, status);
  TORCH_CHECK(p.N == J * H * D, "gemm_headmajor: N must equal J*H*D");
  TORCH_CHECK(p.M % (T * n_rows) == 0, "gemm_headmajor: M must be a multiple of T*n_rows");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() &&
                  out.numel() == (p.M / (T * n_rows)) * T * J * H * n_rows * Dp,
              "gemm_headmajor: contiguous bf16 output of the head-major size expected");
  if (p.M == 0) return;
  p.out = out.data_ptr();
  p.row_scale = opt_f32(row_scale, p.M, "row_scale");
  p.hm = HeadMajorMap{static_cast<int>(T), static_cast<int>(n_rows), static_cast<int>(J), static_cast<int>(H),
                      static_cast<int>(D), static_cast<int>(Dp)};
  dispatch_bn<kHeadMajor>(bn > 0 ? static_cast<int>(bn) : choose_bn(p.N), A, B, p, at::cuda::getCurrentCUDAStream());
}

}  // namespace nori
