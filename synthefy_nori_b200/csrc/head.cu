// Row-wise LayerNorm fused with an activation, its backward, and bias-gradient column
// sums: the memory-bound pieces between the tcgen05 GEMMs of the regression head
// (E -> LN -> Linear -> LN -> GELU -> Linear -> 999 quantiles) and of the embedding
// MLPs.  One warp owns one row (C <= 2048 values held in registers, 64 per lane), so a
// row is read once and written once in each direction.
//
// Reference counterparts: torch LayerNorm + GELU / ReLU inside reg_y_decoder
// (model/transformer.py:345-350) and the encoder's fusion MLP (model/encoders.py:
// 432-585), and the bias gradients autograd computes for their Linear layers.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>

#include "sm100.cuh"

namespace nori {

enum Act : int { kActNone = 0, kActGelu = 1, kActRelu = 2 };
constexpr int kLnMaxPerLane = 64;  // C <= 2048

__device__ __forceinline__ float act_fwd(float z, int act) {
  if (act == kActGelu) return 0.5f * z * (1.f + erff(z * 0.70710678118654752f));
  if (act == kActRelu) return fmaxf(z, 0.f);
  return z;
}

__device__ __forceinline__ float act_grad(float z, int act) {
  if (act == kActGelu) {
    const float cdf = 0.5f * (1.f + erff(z * 0.70710678118654752f));
    const float pdf = 0.3989422804014327f * __expf(-0.5f * z * z);
    return cdf + z * pdf;
  }
  if (act == kActRelu) return z > 0.f ? 1.f : 0.f;
  return 1.f;
}

template <typename T>
__device__ __forceinline__ float ld_as_f32(const T* p);
template <>
__device__ __forceinline__ float ld_as_f32<float>(const float* p) {
  return *p;
}
template <>
__device__ __forceinline__ float ld_as_f32<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

// y = act(gamma * (x - mean) * rstd + beta); x rows strided by ldx, y contiguous [R, C].
template <typename T>
__global__ void ln_act_fwd_kernel(const T* __restrict__ x, int64_t ldx, int64_t R, int C,
                                  const float* __restrict__ gamma, const float* __restrict__ beta, float eps, int act,
                                  __nv_bfloat16* __restrict__ y, float* __restrict__ mean_out,
                                  float* __restrict__ rstd_out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= R) return;
  const T* xr = x + row * ldx;
  float v[kLnMaxPerLane];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kLnMaxPerLane; ++i) {
    const int c = lane + 32 * i;
    v[i] = c < C ? ld_as_f32(xr + c) : 0.f;
    s += v[i];
  }
  const float mean = warp_sum(s) / static_cast<float>(C);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kLnMaxPerLane; ++i) {
    const int c = lane + 32 * i;
    const float d = c < C ? v[i] - mean : 0.f;
    ss += d * d;
  }
  const float rstd = rsqrtf(warp_sum(ss) / static_cast<float>(C) + eps);
  __nv_bfloat16* yr = y + row * static_cast<int64_t>(C);
#pragma unroll
  for (int i = 0; i < kLnMaxPerLane; ++i) {
    const int c = lane + 32 * i;
    if (c < C) {
      const float z = (v[i] - mean) * rstd * (gamma ? gamma[c] : 1.f) + (beta ? beta[c] : 0.f);
      yr[c] = __float2bfloat16(act_fwd(z, act));
    }
  }
  if (lane == 0) {
    mean_out[row] = mean;
    rstd_out[row] = rstd;
  }
}

// Backward of ln_act_fwd: dx (rows strided by lddx, bf16), dgamma / dbeta accumulated
// (fp32, += ; per-CTA partial sums in shared memory, then one atomic per column).
template <typename T>
__global__ void ln_act_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const T* __restrict__ x, int64_t ldx,
                                  int64_t R, int C, const float* __restrict__ gamma, const float* __restrict__ beta,
                                  const float* __restrict__ mean_in, const float* __restrict__ rstd_in, int act,
                                  __nv_bfloat16* __restrict__ dx, int64_t lddx, float* __restrict__ dgamma,
                                  float* __restrict__ dbeta) {
  extern __shared__ float sh[];  // [2 * C]: dgamma, dbeta partials of this CTA
  float* sg = sh;
  float* sb = sh + C;
  for (int c = threadIdx.x; c < 2 * C; c += blockDim.x) sh[c] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x / 32;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * warps + (threadIdx.x >> 5); row < R;
       row += static_cast<int64_t>(gridDim.x) * warps) {
    const T* xr = x + row * ldx;
    const __nv_bfloat16* dyr = dy + row * static_cast<int64_t>(C);
    const float mean = mean_in[row], rstd = rstd_in[row];
    float dxh[kLnMaxPerLane];  // x-hat is recomputed in the second pass (fewer live registers)
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < kLnMaxPerLane; ++i) {
      const int c = lane + 32 * i;
      dxh[i] = 0.f;
      if (c < C) {
        const float g = gamma ? gamma[c] : 1.f;
        const float xh = (ld_as_f32(xr + c) - mean) * rstd;
        const float z = xh * g + (beta ? beta[c] : 0.f);
        const float dz = __bfloat162float(dyr[c]) * act_grad(z, act);
        atomicAdd(&sg[c], dz * xh);
        atomicAdd(&sb[c], dz);
        dxh[i] = dz * g;
        s1 += dxh[i];
        s2 += dxh[i] * xh;
      }
    }
    s1 = warp_sum(s1) / static_cast<float>(C);
    s2 = warp_sum(s2) / static_cast<float>(C);
    __nv_bfloat16* dxr = dx + row * lddx;
#pragma unroll
    for (int i = 0; i < kLnMaxPerLane; ++i) {
      const int c = lane + 32 * i;
      if (c < C) {
        const float xh = (ld_as_f32(xr + c) - mean) * rstd;
        dxr[c] = __float2bfloat16(rstd * (dxh[i] - s1 - xh * s2));
      }
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    if (dgamma) atomicAdd(&dgamma[c], sg[c]);
    if (dbeta) atomicAdd(&dbeta[c], sb[c]);
  }
}

// out[c] += sum_r y[r, c] for c < N (bf16 rows strided by ld): the bias gradient.
__global__ void colsum_kernel(const __nv_bfloat16* __restrict__ y, int64_t ld, int64_t R, int N, int rows_per_cta,
                              float* __restrict__ out) {
  const int c = blockIdx.y * blockDim.x + threadIdx.x;
  if (c >= N) return;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_cta;
  const int64_t r1 = r0 + rows_per_cta < R ? r0 + rows_per_cta : R;
  float s = 0.f;
  for (int64_t r = r0; r < r1; ++r) s += __bfloat162float(y[r * ld + c]);
  atomicAdd(&out[c], s);
}

// Vectorised variants (bf16 rows, C a multiple of 8, 16-byte aligned rows): each lane
// owns CH chunks of 8 consecutive columns (16-byte loads / stores); the backward keeps
// its columns' dgamma / dbeta partial sums in registers across all rows the warp visits
// and reduces them once per CTA.
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float* v) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

template <int CH>
__global__ void ln_act_fwd_vec_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int64_t R, int C,
                                      const float* __restrict__ gamma, const float* __restrict__ beta, float eps,
                                      int act, __nv_bfloat16* __restrict__ y, float* __restrict__ mean_out,
                                      float* __restrict__ rstd_out) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * warps + (threadIdx.x >> 5); row < R;
       row += static_cast<int64_t>(gridDim.x) * warps) {
    const __nv_bfloat16* xr = x + row * ldx;
    float v[CH * 8];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < CH; ++j) {
      const int c0 = 8 * (lane + 32 * j);
      if (c0 < C) {
        load8(xr + c0, v + 8 * j);
#pragma unroll
        for (int i = 0; i < 8; ++i) s += v[8 * j + i];
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[8 * j + i] = 0.f;
      }
    }
    const float mean = warp_sum(s) / static_cast<float>(C);
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < CH; ++j) {
      if (8 * (lane + 32 * j) < C) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float d = v[8 * j + i] - mean;
          ss += d * d;
        }
      }
    }
    const float rstd = rsqrtf(warp_sum(ss) / static_cast<float>(C) + eps);
    __nv_bfloat16* yr = y + row * static_cast<int64_t>(C);
#pragma unroll
    for (int j = 0; j < CH; ++j) {
      const int c0 = 8 * (lane + 32 * j);
      if (c0 < C) {
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float z = (v[8 * j + i] - mean) * rstd * (gamma ? gamma[c0 + i] : 1.f) + (beta ? beta[c0 + i] : 0.f);
          o[i] = act_fwd(z, act);
        }
        store8(yr + c0, o);
      }
    }
    if (lane == 0) {
      mean_out[row] = mean;
      rstd_out[row] = rstd;
    }
  }
}

template <int CH>
__global__ void ln_act_bwd_vec_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                      int64_t ldx, int64_t R, int C, const float* __restrict__ gamma,
                                      const float* __restrict__ beta, const float* __restrict__ mean_in,
                                      const float* __restrict__ rstd_in, int act, __nv_bfloat16* __restrict__ dx,
                                      int64_t lddx, float* __restrict__ dgamma, float* __restrict__ dbeta) {
  extern __shared__ float sh[];  // [2 * C]
  for (int c = threadIdx.x; c < 2 * C; c += blockDim.x) sh[c] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  float gacc[CH * 8], bacc[CH * 8];
#pragma unroll
  for (int i = 0; i < CH * 8; ++i) gacc[i] = bacc[i] = 0.f;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * warps + (threadIdx.x >> 5); row < R;
       row += static_cast<int64_t>(gridDim.x) * warps) {
    const __nv_bfloat16* xr = x + row * ldx;
    const __nv_bfloat16* dyr = dy + row * static_cast<int64_t>(C);
    const float mean = mean_in[row], rstd = rstd_in[row];
    float s1 = 0.f, s2 = 0.f;
    // pass 1: column partial sums (registers) and the two row reductions
#pragma unroll
    for (int j = 0; j < CH; ++j) {
      const int c0 = 8 * (lane + 32 * j);
      if (c0 < C) {
        float xv[8], gv[8];
        load8(xr + c0, xv);
        load8(dyr + c0, gv);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float g = gamma ? gamma[c0 + i] : 1.f;
          const float h = (xv[i] - mean) * rstd;
          const float dz = gv[i] * act_grad(h * g + (beta ? beta[c0 + i] : 0.f), act);
          gacc[8 * j + i] += dz * h;
          bacc[8 * j + i] += dz;
          s1 += dz * g;
          s2 += dz * g * h;
        }
      }
    }
    s1 = warp_sum(s1) / static_cast<float>(C);
    s2 = warp_sum(s2) / static_cast<float>(C);
    // pass 2: the row (still in L1) again, dx written
    __nv_bfloat16* dxr = dx + row * lddx;
#pragma unroll
    for (int j = 0; j < CH; ++j) {
      const int c0 = 8 * (lane + 32 * j);
      if (c0 < C) {
        float xv[8], gv[8], o[8];
        load8(xr + c0, xv);
        load8(dyr + c0, gv);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float g = gamma ? gamma[c0 + i] : 1.f;
          const float h = (xv[i] - mean) * rstd;
          const float dz = gv[i] * act_grad(h * g + (beta ? beta[c0 + i] : 0.f), act);
          o[i] = rstd * (dz * g - s1 - h * s2);
        }
        store8(dxr + c0, o);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const int c0 = 8 * (lane + 32 * j);
    if (c0 < C) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        atomicAdd(&sh[c0 + i], gacc[8 * j + i]);
        atomicAdd(&sh[C + c0 + i], bacc[8 * j + i]);
      }
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    if (dgamma) atomicAdd(&dgamma[c], sh[c]);
    if (dbeta) atomicAdd(&dbeta[c], sh[C + c]);
  }
}

static bool vec_ok(const torch::Tensor& t) {
  return t.scalar_type() == at::kBFloat16 && t.size(1) % 8 == 0 && t.stride(0) % 8 == 0 &&
         reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0;
}

// ------------------------------------------------------------------ host
static void check_vec(const c10::optional<torch::Tensor>& t, int64_t n, const char* what) {
  if (!t.has_value() || !t->defined()) return;
  TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == n, what,
              ": contiguous fp32 vector of the row width expected");
}

static const float* opt_ptr(const c10::optional<torch::Tensor>& t) {
  return t.has_value() && t->defined() ? t->data_ptr<float>() : nullptr;
}

// x: [R, C] with row stride x.stride(0) (unit column stride), bf16 or fp32.
std::vector<torch::Tensor> ln_act_fwd(const torch::Tensor& x, const c10::optional<torch::Tensor>& gamma,
                                      const c10::optional<torch::Tensor>& beta, double eps, int64_t act) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.stride(1) == 1, "ln_act_fwd: [R, C] rows with unit column stride");
  const int64_t R = x.size(0);
  const int C = static_cast<int>(x.size(1));
  TORCH_CHECK(C >= 1 && C <= 32 * kLnMaxPerLane, "ln_act_fwd: 1 <= C <= 2048");
  TORCH_CHECK(act >= 0 && act <= 2, "ln_act_fwd: act 0 (none), 1 (gelu), 2 (relu)");
  check_vec(gamma, C, "gamma");
  check_vec(beta, C, "beta");
  const at::cuda::CUDAGuard guard(x.device());
  auto y = torch::empty({R, C}, x.options().dtype(at::kBFloat16));
  auto mean = torch::empty({R}, x.options().dtype(at::kFloat));
  auto rstd = torch::empty({R}, x.options().dtype(at::kFloat));
  if (R == 0) return {y, mean, rstd};
  const int warps = 8;
  const unsigned blocks = static_cast<unsigned>((R + warps - 1) / warps);
  auto s = at::cuda::getCurrentCUDAStream();
  auto* yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  if (vec_ok(x)) {
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, x.get_device());
    const unsigned vb = static_cast<unsigned>(std::min<int64_t>((R + warps - 1) / warps, 16 * std::max(sms, 1)));
    auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
    const float* gp = opt_ptr(gamma);
    const float* bp = opt_ptr(beta);
    const int a = static_cast<int>(act);
    const float e = static_cast<float>(eps);
    const int ch = (C + 255) / 256;
    if (ch == 6)
      ln_act_fwd_vec_kernel<6><<<vb, 256, 0, s>>>(xp, x.stride(0), R, C, gp, bp, e, a, yp, mean.data_ptr<float>(), rstd.data_ptr<float>());
    else if (ch <= 1)
      ln_act_fwd_vec_kernel<1><<<vb, 256, 0, s>>>(xp, x.stride(0), R, C, gp, bp, e, a, yp, mean.data_ptr<float>(), rstd.data_ptr<float>());
    else if (ch <= 2)
      ln_act_fwd_vec_kernel<2><<<vb, 256, 0, s>>>(xp, x.stride(0), R, C, gp, bp, e, a, yp, mean.data_ptr<float>(), rstd.data_ptr<float>());
    else if (ch <= 4)
      ln_act_fwd_vec_kernel<4><<<vb, 256, 0, s>>>(xp, x.stride(0), R, C, gp, bp, e, a, yp, mean.data_ptr<float>(), rstd.data_ptr<float>());
    else
      ln_act_fwd_vec_kernel<8><<<vb, 256, 0, s>>>(xp, x.stride(0), R, C, gp, bp, e, a, yp, mean.data_ptr<float>(), rstd.data_ptr<float>());
  } else if (x.scalar_type() == at::kBFloat16) {
    ln_act_fwd_kernel<__nv_bfloat16><<<blocks, 32 * warps, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), R, C, opt_ptr(gamma), opt_ptr(beta),
        static_cast<float>(eps), static_cast<int>(act), yp, mean.data_ptr<float>(), rstd.data_ptr<float>());
  } else {
    TORCH_CHECK(x.scalar_type() == at::kFloat, "ln_act_fwd: bf16 or fp32 input");
    ln_act_fwd_kernel<float><<<blocks, 32 * warps, 0, s>>>(x.data_ptr<float>(), x.stride(0), R, C, opt_ptr(gamma),
                                                           opt_ptr(beta), static_cast<float>(eps), static_cast<int>(act),
                                                           yp, mean.data_ptr<float>(), rstd.data_ptr<float>());
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {y, mean, rstd};
}

// dy: contiguous bf16 [R, C]; dx: bf16 [R, C] (row stride dx.stride(0)); dgamma / dbeta: fp32 [C], accumulated.
void ln_act_bwd(const torch::Tensor& dy, const torch::Tensor& x, const c10::optional<torch::Tensor>& gamma,
                const c10::optional<torch::Tensor>& beta, const torch::Tensor& mean, const torch::Tensor& rstd,
                int64_t act, torch::Tensor& dx, const c10::optional<torch::Tensor>& dgamma,
                const c10::optional<torch::Tensor>& dbeta) {
  TORCH_CHECK(dy.is_cuda() && dy.scalar_type() == at::kBFloat16 && dy.is_contiguous() && dy.dim() == 2,
              "ln_act_bwd: contiguous bf16 dy [R, C]");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && x.size(0) == dy.size(0) && x.size(1) == dy.size(1),
              "ln_act_bwd: x [R, C] with unit column stride");
  TORCH_CHECK(dx.scalar_type() == at::kBFloat16 && dx.dim() == 2 && dx.stride(1) == 1 && dx.size(0) == dy.size(0) &&
                  dx.size(1) == dy.size(1),
              "ln_act_bwd: bf16 dx [R, C] with unit column stride");
  const int64_t R = dy.size(0);
  const int C = static_cast<int>(dy.size(1));
  TORCH_CHECK(C >= 1 && C <= 32 * kLnMaxPerLane, "ln_act_bwd: 1 <= C <= 2048");
  check_vec(gamma, C, "gamma");
  check_vec(beta, C, "beta");
  check_vec(dgamma, C, "dgamma");
  check_vec(dbeta, C, "dbeta");
  TORCH_CHECK(mean.numel() == R && rstd.numel() == R, "ln_act_bwd: per-row mean / rstd");
  const at::cuda::CUDAGuard guard(dy.device());
  if (R == 0) return;
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dy.get_device());
  const int warps = 8;
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((R + warps - 1) / warps, 4 * std::max(sms, 1)));
  const size_t smem = 2 * static_cast<size_t>(C) * sizeof(float);
  auto s = at::cuda::getCurrentCUDAStream();
  auto* dyp = reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr());
  auto* dxp = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
  if (vec_ok(x) && vec_ok(dx) && vec_ok(dy)) {
    auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
    const float *gp = opt_ptr(gamma), *bp = opt_ptr(beta);
    float *dgp = const_cast<float*>(opt_ptr(dgamma)), *dbp = const_cast<float*>(opt_ptr(dbeta));
    const int a = static_cast<int>(act);
    const int ch = (C + 255) / 256;
    if (ch == 6)
      ln_act_bwd_vec_kernel<6><<<blocks, 32 * warps, smem, s>>>(dyp, xp, x.stride(0), R, C, gp, bp, mean.data_ptr<float>(), rstd.data_ptr<float>(), a, dxp, dx.stride(0), dgp, dbp);
    else if (ch <= 1)
      ln_act_bwd_vec_kernel<1><<<blocks, 32 * warps, smem, s>>>(dyp, xp, x.stride(0), R, C, gp, bp, mean.data_ptr<float>(), rstd.data_ptr<float>(), a, dxp, dx.stride(0), dgp, dbp);
    else if (ch <= 2)
      ln_act_bwd_vec_kernel<2><<<blocks, 32 * warps, smem, s>>>(dyp, xp, x.stride(0), R, C, gp, bp, mean.data_ptr<float>(), rstd.data_ptr<float>(), a, dxp, dx.stride(0), dgp, dbp);
    else if (ch <= 4)
      ln_act_bwd_vec_kernel<4><<<blocks, 32 * warps, smem, s>>>(dyp, xp, x.stride(0), R, C, gp, bp, mean.data_ptr<float>(), rstd.data_ptr<float>(), a, dxp, dx.stride(0), dgp, dbp);
    else
      ln_act_bwd_vec_kernel<8><<<blocks, 32 * warps, smem, s>>>(dyp, xp, x.stride(0), R, C, gp, bp, mean.data_ptr<float>(), rstd.data_ptr<float>(), a, dxp, dx.stride(0), dgp, dbp);
  } else if (x.scalar_type() == at::kBFloat16) {
    ln_act_bwd_kernel<__nv_bfloat16><<<blocks, 32 * warps, smem, s>>>(
        dyp, reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), R, C, opt_ptr(gamma), opt_ptr(beta),
        mean.data_ptr<float>(), rstd.data_ptr<float>(), static_cast<int>(act), dxp, dx.stride(0),
        const_cast<float*>(opt_ptr(dgamma)), const_cast<float*>(opt_ptr(dbeta)));
  } else {
    TORCH_CHECK(x.scalar_type() == at::kFloat, "ln_act_bwd: bf16 or fp32 input");
    ln_act_bwd_kernel<float><<<blocks, 32 * warps, smem, s>>>(
        dyp, x.data_ptr<float>(), x.stride(0), R, C, opt_ptr(gamma), opt_ptr(beta), mean.data_ptr<float>(),
        rstd.data_ptr<float>(), static_cast<int>(act), dxp, dx.stride(0), const_cast<float*>(opt_ptr(dgamma)),
        const_cast<float*>(opt_ptr(dbeta)));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// out[c] += sum_r y[r, c] for c < out.numel(); y bf16 [R, >= N] with unit column stride.
void colsum_bf16(const torch::Tensor& y, torch::Tensor& out) {
  TORCH_CHECK(y.is_cuda() && y.scalar_type() == at::kBFloat16 && y.dim() == 2 && y.stride(1) == 1,
              "colsum: bf16 [R, N] with unit column stride");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() <= y.size(1), "colsum: fp32 out");
  const at::cuda::CUDAGuard guard(y.device());
  const int64_t R = y.size(0);
  const int N = static_cast<int>(out.numel());
  if (R == 0 || N == 0) return;
  const int rows_per_cta = 64;
  const dim3 grid(static_cast<unsigned>((R + rows_per_cta - 1) / rows_per_cta), static_cast<unsigned>((N + 255) / 256));
  TORCH_CHECK(grid.x < 2147483647u, "colsum: too many rows");
  colsum_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), y.stride(0), R, N, rows_per_cta, out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace nori

namespace nori {

// Online merge of one attention partial into a running result, for queries that attend
// to a context streamed in row blocks: with m = max(lse_acc, lse_b),
//   acc <- (e^(lse_acc - m) acc + e^(lse_b - m) o_b) / (e^(lse_acc - m) + e^(lse_b - m)),
//   lse_acc <- m + log(e^(lse_acc - m) + e^(lse_b - m)).
// acc fp32 [R, E] (query token rows), o_b bf16 [R, E]; lse [B T H, nq] in the sequence
// attention's (table, token, head)-major order; row r = (b nq + s) T + t, head h of row r
// has lse index ((b T + t) H + h) nq + s.  first != 0 initialises acc / lse_acc.
__global__ void attn_lse_merge_kernel(float* __restrict__ acc, float* __restrict__ lse_acc,
                                      const __nv_bfloat16* __restrict__ ob, const float* __restrict__ lse_b,
                                      int64_t R, int T, int H, int D, int nq, int first) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // (row, head)
  if (i >= R * H) return;
  const int64_t r = i / H;
  const int h = static_cast<int>(i % H);
  const int t = static_cast<int>(r % T);
  const int64_t bs = r / T;
  const int s = static_cast<int>(bs % nq);
  const int64_t b = bs / nq;
  const int64_t li = ((b * T + t) * H + h) * nq + s;
  float* a = acc + r * static_cast<int64_t>(H) * D + static_cast<int64_t>(h) * D;
  const __nv_bfloat16* o = ob + r * static_cast<int64_t>(H) * D + static_cast<int64_t>(h) * D;
  const float lb = lse_b[li];
  if (first) {
    for (int d = 0; d < D; ++d) a[d] = __bfloat162float(o[d]);
    lse_acc[li] = lb;
    return;
  }
  const float la = lse_acc[li];
  const float m = fmaxf(la, lb);
  if (m == -INFINITY) return;
  const float wa = __expf(la - m), wb = __expf(lb - m);
  const float inv = 1.f / (wa + wb);
  for (int d = 0; d < D; ++d) a[d] = (wa * a[d] + wb * __bfloat162float(o[d])) * inv;
  lse_acc[li] = m + __logf(wa + wb);
}

void attn_lse_merge(torch::Tensor& acc, torch::Tensor& lse_acc, const torch::Tensor& ob, const torch::Tensor& lse_b,
                    int64_t T, int64_t H, int64_t nq, bool first) {
  TORCH_CHECK(acc.is_cuda() && acc.scalar_type() == at::kFloat && acc.is_contiguous() && acc.dim() == 2,
              "attn_lse_merge: contiguous fp32 acc [R, E]");
  TORCH_CHECK(ob.scalar_type() == at::kBFloat16 && ob.is_contiguous() && ob.sizes() == acc.sizes(),
              "attn_lse_merge: contiguous bf16 partial [R, E]");
  TORCH_CHECK(lse_acc.scalar_type() == at::kFloat && lse_b.scalar_type() == at::kFloat && lse_acc.is_contiguous() &&
                  lse_b.is_contiguous() && lse_acc.numel() == lse_b.numel() && lse_b.numel() == acc.size(0) * H,
              "attn_lse_merge: fp32 lse [B T H, nq] for both");
  const int64_t R = acc.size(0);
  TORCH_CHECK(H > 0 && acc.size(1) % H == 0 && T > 0 && nq > 0 && R % (T * nq) == 0, "attn_lse_merge: shapes");
  const at::cuda::CUDAGuard guard(acc.device());
  if (R == 0) return;
  const int64_t n = R * H;
  attn_lse_merge_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      acc.data_ptr<float>(), lse_acc.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(ob.data_ptr()),
      lse_b.data_ptr<float>(), R, static_cast<int>(T), static_cast<int>(H), static_cast<int>(acc.size(1) / H),
      static_cast<int>(nq), first ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace nori
