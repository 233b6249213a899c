// Memory-bound kernels of the Nori step: RMS row scales, the fused 999-quantile
// pinball objective (forward value and gradient in one pass), the gradient-norm
// reduction, the fused AdamW + EMA + bf16 weight refresh, and the per-(row, head)
// int8 KV quantizer.
//
// Reference semantics:
//   RMSNorm without affine weight  model/layer.py:233-258
//   pinball objective              training/loss.py:45-106, 363-575 (per-episode mean,
//                                  monotonicity penalty, aux MSE / per-episode variance)
//   grad clip 1.0 + AdamW + EMA    training/trainer.py:1544-1552, 38-63
//   int8 KV quantization           model/kv_cache_scaling.py:29-41
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "sm100.cuh"

namespace nori {

// ------------------------------------------------------------------ RMS row scale
// rs[m] = rsqrt(mean(x[m, :]^2) + eps); one warp per row, 16-byte loads.
__global__ void rms_scale_kernel(const __nv_bfloat16* __restrict__ x, int64_t M, int E, int64_t ld, float eps,
                                 float* __restrict__ rs) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= M) return;
  const __nv_bfloat16* xr = x + row * ld;
  float s = 0.f;
  if ((E % 8) == 0) {
    for (int c = lane * 8; c < E; c += 256) {
      uint4 w = *reinterpret_cast<const uint4*>(xr + c);
      uint32_t a[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float lo = bf16lo(a[i]), hi = bf16hi(a[i]);
        s += lo * lo + hi * hi;
      }
    }
  } else {
    for (int c = lane; c < E; c += 32) {
      const float v = __bfloat162float(xr[c]);
      s += v * v;
    }
  }
  s = warp_sum(s);
  if (lane == 0) rs[row] = rsqrtf(s / static_cast<float>(E) + eps);
}

torch::Tensor rms_scale(const torch::Tensor& x, double eps) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1,
              "rms_scale: bf16 [M, E] row-major input expected");
  const at::cuda::CUDAGuard guard(x.device());
  auto rs = torch::empty({x.size(0)}, x.options().dtype(at::kFloat));
  const int64_t M = x.size(0);
  if (M == 0) return rs;
  TORCH_CHECK(x.size(1) % 8 != 0 || (x.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0),
              "rms_scale: 16-byte aligned rows expected");
  const int warps = 8;
  rms_scale_kernel<<<(M + warps - 1) / warps, warps * 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), M, static_cast<int>(x.size(1)), x.stride(0),
      static_cast<float>(eps), rs.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return rs;
}

// xn = bf16(x * rs[row]); one warp per row.
__global__ void rms_apply_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ rs, int64_t M, int E,
                                 __nv_bfloat16* __restrict__ y) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= M) return;
  const float r = rs[row];
  const __nv_bfloat16* xr = x + row * E;
  __nv_bfloat16* yr = y + row * E;
  for (int c = lane * 8; c < E; c += 256) {
    const uint4 w = *reinterpret_cast<const uint4*>(xr + c);
    const uint32_t a[4] = {w.x, w.y, w.z, w.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = pack_bf16x2(bf16lo(a[i]) * r, bf16hi(a[i]) * r);
    *reinterpret_cast<uint4*>(yr + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

torch::Tensor rms_apply(const torch::Tensor& x, const torch::Tensor& rs) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.is_contiguous() && x.size(1) % 8 == 0,
              "rms_apply: contiguous bf16 [M, E] (E % 8 == 0)");
  TORCH_CHECK(rs.scalar_type() == at::kFloat && rs.numel() == x.size(0), "rms_apply: fp32 rs [M]");
  const at::cuda::CUDAGuard guard(x.device());
  auto y = torch::empty_like(x);
  const int64_t M = x.size(0);
  if (M == 0) return y;
  rms_apply_kernel<<<(M + 7) / 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), rs.data_ptr<float>(), M, static_cast<int>(x.size(1)),
      reinterpret_cast<__nv_bfloat16*>(y.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return y;
}

// RMSNorm (no affine) backward fused with the residual-gradient add:
//   dx = dres + rs * dxn - x * rs^3 * mean(dxn * x)
__global__ void rms_bwd_kernel(const __nv_bfloat16* __restrict__ dxn, const __nv_bfloat16* __restrict__ x,
                               const float* __restrict__ rs, const __nv_bfloat16* __restrict__ dres, int64_t M, int E,
                               __nv_bfloat16* __restrict__ dx) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= M) return;
  const __nv_bfloat16* gr = dxn + row * E;
  const __nv_bfloat16* xr = x + row * E;
  float dot = 0.f;
  for (int c = lane * 8; c < E; c += 256) {
    const uint4 g = *reinterpret_cast<const uint4*>(gr + c);
    const uint4 w = *reinterpret_cast<const uint4*>(xr + c);
    const uint32_t ga[4] = {g.x, g.y, g.z, g.w}, xa[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) dot += bf16lo(ga[i]) * bf16lo(xa[i]) + bf16hi(ga[i]) * bf16hi(xa[i]);
  }
  dot = warp_sum(dot);
  const float r = rs[row];
  const float coef = r * r * r * dot / static_cast<float>(E);
  for (int c = lane * 8; c < E; c += 256) {
    const uint4 g = *reinterpret_cast<const uint4*>(gr + c);
    const uint4 w = *reinterpret_cast<const uint4*>(xr + c);
    const uint32_t ga[4] = {g.x, g.y, g.z, g.w}, xa[4] = {w.x, w.y, w.z, w.w};
    uint32_t da[4] = {0u, 0u, 0u, 0u};
    if (dres != nullptr) {
      const uint4 d = *reinterpret_cast<const uint4*>(dres + row * E + c);
      da[0] = d.x; da[1] = d.y; da[2] = d.z; da[3] = d.w;
    }
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float lo = bf16lo(da[i]) + r * bf16lo(ga[i]) - coef * bf16lo(xa[i]);
      const float hi = bf16hi(da[i]) + r * bf16hi(ga[i]) - coef * bf16hi(xa[i]);
      o[i] = pack_bf16x2(lo, hi);
    }
    *reinterpret_cast<uint4*>(dx + row * E + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

torch::Tensor rms_bwd(const torch::Tensor& dxn, const torch::Tensor& x, const torch::Tensor& rs,
                      const c10::optional<torch::Tensor>& dres) {
  for (const torch::Tensor* t : std::initializer_list<const torch::Tensor*>{&dxn, &x})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->is_contiguous() && t->sizes() == x.sizes() &&
                    x.dim() == 2 && x.size(1) % 8 == 0,
                "rms_bwd: contiguous bf16 [M, E] (E % 8 == 0)");
  const __nv_bfloat16* dr = nullptr;
  if (dres.has_value() && dres->defined()) {
    TORCH_CHECK(dres->scalar_type() == at::kBFloat16 && dres->is_contiguous() && dres->sizes() == x.sizes(),
                "rms_bwd: dres like x");
    dr = reinterpret_cast<const __nv_bfloat16*>(dres->data_ptr());
  }
  const at::cuda::CUDAGuard guard(x.device());
  auto dx = torch::empty_like(x);
  const int64_t M = x.size(0);
  if (M == 0) return dx;
  rms_bwd_kernel<<<(M + 7) / 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dxn.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
      rs.data_ptr<float>(), dr, M, static_cast<int>(x.size(1)), reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dx;
}

// SwiGLU backward on the interleaved (gate, up) pre-activations:
//   h = silu(g) u ;  dg = dh u silu'(g) ;  du = dh silu(g)
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dh, const __nv_bfloat16* __restrict__ gu,
                                  int64_t n_pairs, __nv_bfloat16* __restrict__ dgu) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n_pairs; i += stride) {
    const uint32_t pr = reinterpret_cast<const uint32_t*>(gu)[i];
    const float g = bf16lo(pr), u = bf16hi(pr);
    const float d = __bfloat162float(dh[i]);
    const float sg = 1.0f / (1.0f + __expf(-g));
    const float dg = d * u * sg * (1.0f + g * (1.0f - sg));
    const float du = d * g * sg;
    reinterpret_cast<uint32_t*>(dgu)[i] = pack_bf16x2(dg, du);
  }
}

torch::Tensor swiglu_bwd(const torch::Tensor& dh, const torch::Tensor& gu) {
  TORCH_CHECK(dh.is_cuda() && dh.scalar_type() == at::kBFloat16 && dh.is_contiguous(), "swiglu_bwd: bf16 dh");
  TORCH_CHECK(gu.scalar_type() == at::kBFloat16 && gu.is_contiguous() && gu.numel() == 2 * dh.numel(),
              "swiglu_bwd: interleaved bf16 gate/up with twice the elements of dh");
  const at::cuda::CUDAGuard guard(dh.device());
  auto dgu = torch::empty_like(gu);
  const int64_t n = dh.numel();
  if (n == 0) return dgu;
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 148 * 32));
  swiglu_bwd_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dh.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()), n,
      reinterpret_cast<__nv_bfloat16*>(dgu.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dgu;
}

// GELU backward from the recomputed pre-activation z: d z = dh (Phi(z) + z phi(z)); eight
// bf16 values per thread (16-byte loads / stores).
__global__ void gelu_bwd_kernel(const uint4* __restrict__ dh, const uint4* __restrict__ z, int64_t n8,
                                uint4* __restrict__ dz) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8; i += stride) {
    const uint4 a = dh[i], b = z[i];
    const uint32_t av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float r[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float zz = e ? bf16hi(bv[k]) : bf16lo(bv[k]);
        const float d = e ? bf16hi(av[k]) : bf16lo(av[k]);
        const float cdf = 0.5f * (1.0f + erff(zz * 0.70710678118654752f));
        const float pdf = 0.3989422804014327f * __expf(-0.5f * zz * zz);
        r[e] = d * (cdf + zz * pdf);
      }
      o[k] = pack_bf16x2(r[0], r[1]);
    }
    dz[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

torch::Tensor gelu_bwd(const torch::Tensor& dh, const torch::Tensor& z) {
  TORCH_CHECK(dh.is_cuda() && dh.scalar_type() == at::kBFloat16 && dh.is_contiguous(), "gelu_bwd: bf16 dh");
  TORCH_CHECK(z.scalar_type() == at::kBFloat16 && z.is_contiguous() && z.numel() == dh.numel(),
              "gelu_bwd: bf16 pre-activation of the same size");
  TORCH_CHECK(dh.numel() % 8 == 0, "gelu_bwd: element count must be a multiple of 8");
  const at::cuda::CUDAGuard guard(dh.device());
  auto dz = torch::empty_like(dh);
  const int64_t n8 = dh.numel() / 8;
  if (n8 == 0) return dz;
  const int blocks = static_cast<int>(std::min<int64_t>((n8 + 255) / 256, 148 * 32));
  gelu_bwd_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint4*>(dh.data_ptr()), reinterpret_cast<const uint4*>(z.data_ptr()), n8,
      reinterpret_cast<uint4*>(dz.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dz;
}

__global__ void sumsq_to_scale_kernel(const float* __restrict__ ssq, int64_t M, float inv_e, float eps,
                                      float* __restrict__ rs) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < M) rs[i] = rsqrtf(ssq[i] * inv_e + eps);
}

torch::Tensor sumsq_to_scale(const torch::Tensor& ssq, int64_t E, double eps) {
  TORCH_CHECK(ssq.is_cuda() && ssq.scalar_type() == at::kFloat && ssq.is_contiguous(), "sumsq_to_scale: fp32");
  const at::cuda::CUDAGuard guard(ssq.device());
  auto rs = torch::empty_like(ssq);
  const int64_t M = ssq.numel();
  if (M == 0) return rs;
  sumsq_to_scale_kernel<<<(M + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      ssq.data_ptr<float>(), M, 1.0f / static_cast<float>(E), static_cast<float>(eps), rs.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return rs;
}

// ------------------------------------------------------------------ pinball objective
// pred [R, K] (bf16 or fp32, row r = (episode b = r / nq, query row)), target [R],
// quantiles [K] ascending, inv_var [B] = 1 / clamp(var_b, 0.01).
// Writes grad [R, K] (same dtype as pred) of the batch-mean objective and adds the
// objective into loss[0]. One CTA of 256 threads per row.
// ldp / ldg: row strides of pred and grad; grad columns [K, kpad) are written as zeros
// (a padded gradient feeds a GEMM whose N was rounded up to a multiple of 8).
template <typename T>
__global__ void pinball_kernel(const T* __restrict__ pred, const float* __restrict__ target,
                               const float* __restrict__ quantiles, const float* __restrict__ inv_var, int64_t R,
                               int K, int nq, int B, float tail_w, float mono_w, float mse_w, T* __restrict__ grad,
                               float* __restrict__ loss, int64_t ldp, int64_t ldg, int kpad) {
  const int64_t r = blockIdx.x;
  if (r >= R) return;
  const int b = static_cast<int>(r / nq);
  const T* p = pred + r * ldp;
  T* g = grad + r * ldg;
  for (int k = K + threadIdx.x; k < kpad; k += blockDim.x) g[k] = static_cast<T>(0.f);
  const float t = target[r];
  const float iv = inv_var[b];
  __shared__ float red[3][8];
  // pass 1: mean of predictions (for the aux MSE term)
  float psum = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) psum += static_cast<float>(p[k]);
  psum = warp_sum(psum);
  if ((threadIdx.x & 31) == 0) red[0][threadIdx.x >> 5] = psum;
  __syncthreads();
  float pmean = 0.f;
  for (int w = 0; w < static_cast<int>(blockDim.x / 32); ++w) pmean += red[0][w];
  pmean /= static_cast<float>(K);
  const float s_pin = 1.0f / (static_cast<float>(B) * nq * K);
  const float s_mono = K > 1 ? mono_w / (static_cast<float>(B) * nq * (K - 1)) : 0.f;
  const float s_mse = mse_w / (static_cast<float>(B) * nq);
  const float dm = pmean - t;
  float l_pin = 0.f, l_mono = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const float pk = static_cast<float>(p[k]);
    const float tau = quantiles[k];
    const float w = tail_w > 0.f ? 1.0f + tail_w * 2.0f * fabsf(tau - 0.5f) : 1.0f;
    const float e = t - pk;
    float gk;
    if (e > 0.f) {
      l_pin += w * tau * e;
      gk = -tau;
    } else if (e < 0.f) {
      l_pin += w * (tau - 1.0f) * e;
      gk = 1.0f - tau;
    } else {
      gk = 0.5f - tau;  // torch.maximum splits the gradient on ties
    }
    gk *= w * s_pin;
    if (mono_w > 0.f) {
      if (k + 1 < K) {
        const float d = pk - static_cast<float>(p[k + 1]);
        if (d > 0.f) {
          l_mono += d * d;
          gk += 2.0f * d * s_mono;
        }
      }
      if (k > 0) {
        const float d = static_cast<float>(p[k - 1]) - pk;
        if (d > 0.f) gk -= 2.0f * d * s_mono;
      }
    }
    if (mse_w > 0.f) gk += 2.0f * dm * iv * s_mse / static_cast<float>(K);
    g[k] = static_cast<T>(gk);
  }
  l_pin = warp_sum(l_pin);
  l_mono = warp_sum(l_mono);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) {
    red[1][threadIdx.x >> 5] = l_pin;
    red[2][threadIdx.x >> 5] = l_mono;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = 0.f, m = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x / 32); ++w) {
      a += red[1][w];
      m += red[2][w];
    }
    float total = a * s_pin + m * s_mono;
    if (mse_w > 0.f) total += dm * dm * iv * s_mse;
    atomicAdd(loss, total);
  }
}

// Returns (loss [1] fp32, grad like pred).
std::vector<torch::Tensor> pinball_fused(const torch::Tensor& pred, const torch::Tensor& target,
                                         const torch::Tensor& quantiles, const torch::Tensor& inv_var, int64_t nq,
                                         double tail_w, double mono_w, double mse_w) {
  TORCH_CHECK(pred.is_cuda() && pred.dim() == 2 && pred.is_contiguous(), "pinball: contiguous [R, K] pred");
  TORCH_CHECK(target.scalar_type() == at::kFloat && target.is_contiguous() && target.numel() == pred.size(0),
              "pinball: fp32 target [R]");
  TORCH_CHECK(quantiles.scalar_type() == at::kFloat && quantiles.numel() == pred.size(1), "pinball: fp32 quantiles [K]");
  TORCH_CHECK(inv_var.scalar_type() == at::kFloat && inv_var.is_contiguous(), "pinball: fp32 inv_var [B]");
  TORCH_CHECK(nq > 0 && pred.size(0) % nq == 0 && inv_var.numel() == pred.size(0) / nq, "pinball: R = B * nq");
  const at::cuda::CUDAGuard guard(pred.device());
  auto grad = torch::empty_like(pred);
  auto loss = torch::zeros({1}, pred.options().dtype(at::kFloat));
  const int64_t R = pred.size(0);
  if (R == 0) return {loss, grad};
  const int K = static_cast<int>(pred.size(1));
  const int B = static_cast<int>(R / nq);
  auto s = at::cuda::getCurrentCUDAStream();
  if (pred.scalar_type() == at::kBFloat16) {
    pinball_kernel<__nv_bfloat16><<<R, 256, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(pred.data_ptr()), target.data_ptr<float>(),
        quantiles.data_ptr<float>(), inv_var.data_ptr<float>(), R, K, static_cast<int>(nq), B,
        static_cast<float>(tail_w), static_cast<float>(mono_w), static_cast<float>(mse_w),
        reinterpret_cast<__nv_bfloat16*>(grad.data_ptr()), loss.data_ptr<float>(), K, K, K);
  } else {
    TORCH_CHECK(pred.scalar_type() == at::kFloat, "pinball: bf16 or fp32 pred");
    pinball_kernel<float><<<R, 256, 0, s>>>(pred.data_ptr<float>(), target.data_ptr<float>(),
                                            quantiles.data_ptr<float>(), inv_var.data_ptr<float>(), R, K,
                                            static_cast<int>(nq), B, static_cast<float>(tail_w),
                                            static_cast<float>(mono_w), static_cast<float>(mse_w),
                                            grad.data_ptr<float>(), loss.data_ptr<float>(), K, K, K);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {loss, grad};
}

// Strided bf16 variant for the native head: pred [R, >= K] (row stride pred.stride(0)),
// grad written into a preallocated bf16 [R, kpad] (columns >= K zeroed); returns the loss.
torch::Tensor pinball_fused_into(const torch::Tensor& pred, int64_t K, const torch::Tensor& target,
                                 const torch::Tensor& quantiles, const torch::Tensor& inv_var, int64_t nq,
                                 double tail_w, double mono_w, double mse_w, torch::Tensor& grad) {
  TORCH_CHECK(pred.is_cuda() && pred.scalar_type() == at::kBFloat16 && pred.dim() == 2 && pred.stride(1) == 1 &&
                  pred.size(1) >= K,
              "pinball_into: bf16 [R, >= K] pred with unit column stride");
  TORCH_CHECK(grad.scalar_type() == at::kBFloat16 && grad.is_contiguous() && grad.dim() == 2 &&
                  grad.size(0) == pred.size(0) && grad.size(1) >= K,
              "pinball_into: contiguous bf16 grad [R, kpad >= K]");
  TORCH_CHECK(target.scalar_type() == at::kFloat && target.is_contiguous() && target.numel() == pred.size(0),
              "pinball_into: fp32 target [R]");
  TORCH_CHECK(quantiles.scalar_type() == at::kFloat && quantiles.numel() == K, "pinball_into: fp32 quantiles [K]");
  TORCH_CHECK(nq > 0 && pred.size(0) % nq == 0 && inv_var.numel() == pred.size(0) / nq, "pinball_into: R = B * nq");
  const at::cuda::CUDAGuard guard(pred.device());
  auto loss = torch::zeros({1}, pred.options().dtype(at::kFloat));
  const int64_t R = pred.size(0);
  if (R == 0) return loss;
  pinball_kernel<__nv_bfloat16><<<R, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(pred.data_ptr()), target.data_ptr<float>(), quantiles.data_ptr<float>(),
      inv_var.data_ptr<float>(), R, static_cast<int>(K), static_cast<int>(nq), static_cast<int>(R / nq),
      static_cast<float>(tail_w), static_cast<float>(mono_w), static_cast<float>(mse_w),
      reinterpret_cast<__nv_bfloat16*>(grad.data_ptr()), loss.data_ptr<float>(), pred.stride(0), grad.stride(0),
      static_cast<int>(grad.size(1)));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return loss;
}

// ------------------------------------------------------------------ optimizer
__global__ void sumsq_kernel(const float* __restrict__ g, int64_t n, float* __restrict__ out) {
  float s = 0.f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x * 4;
  for (int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4; i < n; i += stride) {
    if (i + 3 < n) {
      const float4 v = *reinterpret_cast<const float4*>(g + i);
      s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    } else {
      for (int64_t j = i; j < n; ++j) s += g[j] * g[j];
    }
  }
  s = warp_sum(s);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) atomicAdd(out, v);
  }
}

// out[0] += sum(g^2) over a flat fp32 buffer
void grad_sumsq(const torch::Tensor& g, torch::Tensor& out) {
  TORCH_CHECK(g.is_cuda() && g.scalar_type() == at::kFloat && g.is_contiguous(), "grad_sumsq: flat fp32");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(g.data_ptr()) % 16 == 0, "grad_sumsq: 16-byte aligned buffer");
  const at::cuda::CUDAGuard guard(g.device());
  const int64_t n = g.numel();
  if (n == 0) return;
  const int blocks = static_cast<int>(std::min<int64_t>((n / 4 + 255) / 256 + 1, 148 * 8));
  sumsq_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(g.data_ptr<float>(), n, out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

struct AdamWArgs {
  float lr, beta1, beta2, eps, wd, bc1, bc2_sqrt, ema_decay, max_norm, grad_scale;
  int use_ema;
};

// One fused pass: g *= clip (from the device-side norm^2) * grad_scale; AdamW update
// (decoupled decay, bias corrected, as torch.optim.AdamW); ema = d ema + (1-d) p;
// bf16 copy of the new weights for the next forward.
__global__ void adamw_ema_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                                 float* __restrict__ v, float* __restrict__ ema, __nv_bfloat16* __restrict__ pbf,
                                 int64_t n, const float* __restrict__ norm_sq, const float* __restrict__ skip,
                                 AdamWArgs a) {
  // a step the trainer decided (on the device) to skip, or one whose gradient norm is not
  // finite, leaves parameters and optimizer state untouched
  if (skip != nullptr && *skip > 0.f) return;
  if (a.max_norm > 0.f && norm_sq != nullptr && !(*norm_sq < INFINITY)) return;
  float scale = a.grad_scale;
  if (a.max_norm > 0.f && norm_sq != nullptr) {
    const float norm = sqrtf(*norm_sq) * a.grad_scale;
    const float c = a.max_norm / (norm + 1e-6f);
    if (c < 1.f) scale *= c;
  }
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float gi = g[i] * scale;
    float pi = p[i];
    pi *= (1.f - a.lr * a.wd);
    const float mi = a.beta1 * m[i] + (1.f - a.beta1) * gi;
    const float vi = a.beta2 * v[i] + (1.f - a.beta2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    const float denom = sqrtf(vi) / a.bc2_sqrt + a.eps;
    pi -= (a.lr / a.bc1) * mi / denom;
    p[i] = pi;
    if (a.use_ema) ema[i] = a.ema_decay * ema[i] + (1.f - a.ema_decay) * pi;
    if (pbf != nullptr) pbf[i] = __float2bfloat16(pi);
  }
}

void adamw_ema(torch::Tensor& p, const torch::Tensor& g, torch::Tensor& m, torch::Tensor& v,
               const c10::optional<torch::Tensor>& ema, const c10::optional<torch::Tensor>& pbf,
               const c10::optional<torch::Tensor>& norm_sq, double lr, double beta1, double beta2, double eps,
               double wd, int64_t step, double ema_decay, double max_norm, double grad_scale,
               const c10::optional<torch::Tensor>& skip) {
  for (const torch::Tensor* t : std::initializer_list<const torch::Tensor*>{&p, &g, &m, &v})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == p.numel(),
                "adamw_ema: flat fp32 buffers of equal size expected");
  const at::cuda::CUDAGuard guard(p.device());
  AdamWArgs a;
  a.lr = static_cast<float>(lr);
  a.beta1 = static_cast<float>(beta1);
  a.beta2 = static_cast<float>(beta2);
  a.eps = static_cast<float>(eps);
  a.wd = static_cast<float>(wd);
  a.bc1 = static_cast<float>(1.0 - std::pow(beta1, static_cast<double>(step)));
  a.bc2_sqrt = static_cast<float>(std::sqrt(1.0 - std::pow(beta2, static_cast<double>(step))));
  a.ema_decay = static_cast<float>(ema_decay);
  a.max_norm = static_cast<float>(max_norm);
  a.grad_scale = static_cast<float>(grad_scale);
  a.use_ema = ema.has_value() && ema->defined() ? 1 : 0;
  float* ema_p = a.use_ema ? ema->data_ptr<float>() : nullptr;
  __nv_bfloat16* pb = nullptr;
  if (pbf.has_value() && pbf->defined()) {
    TORCH_CHECK(pbf->scalar_type() == at::kBFloat16 && pbf->numel() == p.numel() && pbf->is_contiguous(),
                "adamw_ema: bf16 weight copy of equal size");
    pb = reinterpret_cast<__nv_bfloat16*>(pbf->data_ptr());
  }
  const float* ns = norm_sq.has_value() && norm_sq->defined() ? norm_sq->data_ptr<float>() : nullptr;
  const float* sk = nullptr;
  if (skip.has_value() && skip->defined()) {
    TORCH_CHECK(skip->is_cuda() && skip->scalar_type() == at::kFloat && skip->numel() >= 1, "adamw_ema: fp32 skip flag");
    sk = skip->data_ptr<float>();
  }
  const int64_t n = p.numel();
  if (n == 0) return;
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 148 * 16));
  adamw_ema_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), ema_p, pb, n, ns, sk, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------ int8 KV quantizer
// x [R, D] (R = rows x heads, bf16 or fp32) -> q int8 [R, D], scale fp32 [R]
// scale = max(amax, 1e-12) / 127 ; q = clamp(rint(x / scale), -127, 127)
template <typename T>
__global__ void quant_int8_kernel(const T* __restrict__ x, int64_t R, int D, int8_t* __restrict__ q,
                                  float* __restrict__ scale) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (r >= R) return;
  const T* xr = x + r * D;
  float amax = 0.f;
  for (int c = lane; c < D; c += 32) amax = fmaxf(amax, fabsf(static_cast<float>(xr[c])));
  amax = warp_max(amax);
  // torch evaluates `tensor / 127.0` as a multiply by the fp32 reciprocal
  const float s = fmaxf(amax, 1e-12f) * (1.0f / 127.0f);
  for (int c = lane; c < D; c += 32) {
    float v = rintf(static_cast<float>(xr[c]) / s);
    v = fminf(fmaxf(v, -127.f), 127.f);
    q[r * D + c] = static_cast<int8_t>(v);
  }
  if (lane == 0) scale[r] = s;
}

std::vector<torch::Tensor> quantize_int8(const torch::Tensor& x) {
  TORCH_CHECK(x.is_cuda() && x.is_contiguous() && x.dim() >= 1, "quantize_int8: contiguous CUDA tensor");
  const at::cuda::CUDAGuard guard(x.device());
  const int D = static_cast<int>(x.size(-1));
  const int64_t R = x.numel() / std::max(D, 1);
  auto q = torch::empty(x.sizes(), x.options().dtype(at::kChar));
  auto sizes = x.sizes().vec();
  sizes.back() = 1;
  auto sc = torch::empty(sizes, x.options().dtype(at::kFloat));
  if (R == 0) return {q, sc};
  auto s = at::cuda::getCurrentCUDAStream();
  const int warps = 8;
  const int64_t blocks = (R + warps - 1) / warps;
  if (x.scalar_type() == at::kBFloat16) {
    quant_int8_kernel<__nv_bfloat16><<<blocks, warps * 32, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), R, D, q.data_ptr<int8_t>(), sc.data_ptr<float>());
  } else {
    TORCH_CHECK(x.scalar_type() == at::kFloat, "quantize_int8: bf16 or fp32 input");
    quant_int8_kernel<float><<<blocks, warps * 32, 0, s>>>(x.data_ptr<float>(), R, D, q.data_ptr<int8_t>(),
                                                            sc.data_ptr<float>());
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {q, sc};
}

// q int8 [R, D] with scale fp32 [R] -> bf16 [R, D] = bf16(float(q) * scale), the same
// rounding as dequantising in PyTorch (int8 -> fp32 multiply -> bf16). D % 8 == 0: each
// thread converts 8 values (one 8-byte load, one 16-byte store), all under one scale.
__global__ void dequant_int8_kernel(const int8_t* __restrict__ q, const float* __restrict__ scale, int64_t n8, int D,
                                    __nv_bfloat16* __restrict__ out) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = i * 8;
    const float s = __ldg(scale + e / D);
    const int2 raw = __ldg(reinterpret_cast<const int2*>(q + e));
    const int8_t* b = reinterpret_cast<const int8_t*>(&raw);
    uint4 packed;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&packed);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      o2[j] = __floats2bfloat162_rn(static_cast<float>(b[2 * j]) * s, static_cast<float>(b[2 * j + 1]) * s);
    *reinterpret_cast<uint4*>(out + e) = packed;
  }
}

void dequantize_int8(const torch::Tensor& q, const torch::Tensor& scale, torch::Tensor& out) {
  TORCH_CHECK(q.is_cuda() && q.is_contiguous() && q.scalar_type() == at::kChar, "dequantize_int8: contiguous int8 q");
  TORCH_CHECK(scale.is_contiguous() && scale.scalar_type() == at::kFloat, "dequantize_int8: contiguous fp32 scale");
  TORCH_CHECK(out.is_contiguous() && out.scalar_type() == at::kBFloat16 && out.numel() == q.numel(),
              "dequantize_int8: contiguous bf16 output of q's size");
  const int64_t n = q.numel();
  TORCH_CHECK(n == 0 || n % scale.numel() == 0, "dequantize_int8: q rows must match the scales");
  if (n == 0) return;
  const int D = static_cast<int>(n / scale.numel());
  TORCH_CHECK(D % 8 == 0, "dequantize_int8: row length must be a multiple of 8");
  const at::cuda::CUDAGuard guard(q.device());
  const int64_t n8 = n / 8;
  const int blocks = static_cast<int>(std::min<int64_t>((n8 + 255) / 256, 148 * 32));
  dequant_int8_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      q.data_ptr<int8_t>(), scale.data_ptr<float>(), n8, D, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------ quantile collapse
// Per row: sort the K predicted quantiles ascending (monotone quantile function), the
// trapezoid mean of the piecewise-linear quantile function with flat tails
// (tau_0 q_0 + sum 0.5 (q_k + q_{k+1}) dtau + (1 - tau_{K-1}) q_{K-1}), and linear
// interpolation at L requested levels. Reference model/quantile_dist.py:95-208.
// One CTA of 512 threads per row; bitonic sort of up to 1024 values in shared memory.
template <typename T>
__global__ void quantile_decode_kernel(const T* __restrict__ pred, int64_t R, int K, const float* __restrict__ taus,
                                       const float* __restrict__ levels, int L, float* __restrict__ mean,
                                       float* __restrict__ qout, float* __restrict__ sorted_out) {
  __shared__ float v[1024];
  __shared__ float red[16];
  const int64_t r = blockIdx.x;
  if (r >= R) return;
  for (int i = threadIdx.x; i < 1024; i += blockDim.x) v[i] = i < K ? static_cast<float>(pred[r * K + i]) : INFINITY;
  __syncthreads();
  for (int size = 2; size <= 1024; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < 512; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool up = (lo & size) == 0;
        const float a = v[lo], b = v[hi];
        if ((a > b) == up) {
          v[lo] = b;
          v[hi] = a;
        }
      }
      __syncthreads();
    }
  }
  float acc = 0.f;
  for (int k = threadIdx.x; k + 1 < K; k += blockDim.x) acc += 0.5f * (v[k] + v[k + 1]) * (taus[k + 1] - taus[k]);
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x / 32); ++w) tot += red[w];
    tot += taus[0] * v[0] + (1.f - taus[K - 1]) * v[K - 1];
    if (mean != nullptr) mean[r] = tot;
  }
  for (int l = threadIdx.x; l < L; l += blockDim.x) {
    const float t = levels[l];
    float val;
    if (t <= taus[0]) {
      val = v[0];
    } else if (t >= taus[K - 1]) {
      val = v[K - 1];
    } else {
      int lo = 0, hi = K - 1;  // taus[lo] <= t < taus[hi]
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (taus[mid] <= t) lo = mid; else hi = mid;
      }
      const float w = (t - taus[lo]) / (taus[hi] - taus[lo]);
      val = v[lo] + w * (v[hi] - v[lo]);
    }
    qout[r * L + l] = val;
  }
  if (sorted_out != nullptr)
    for (int k = threadIdx.x; k < K; k += blockDim.x) sorted_out[r * K + k] = v[k];
}

// returns (mean [R], quantiles [R, L], sorted [R, K] or empty)
std::vector<torch::Tensor> quantile_decode(const torch::Tensor& pred, const torch::Tensor& taus,
                                           const torch::Tensor& levels, bool return_sorted) {
  TORCH_CHECK(pred.is_cuda() && pred.dim() == 2 && pred.is_contiguous(), "quantile_decode: contiguous [R, K]");
  const int K = static_cast<int>(pred.size(1));
  TORCH_CHECK(K >= 1 && K <= 1024, "quantile_decode: 1 <= K <= 1024");
  TORCH_CHECK(taus.scalar_type() == at::kFloat && taus.numel() == K && taus.is_contiguous(), "quantile_decode: taus");
  TORCH_CHECK(levels.scalar_type() == at::kFloat && levels.is_contiguous(), "quantile_decode: fp32 levels");
  const at::cuda::CUDAGuard guard(pred.device());
  const int64_t R = pred.size(0);
  const int L = static_cast<int>(levels.numel());
  auto fo = pred.options().dtype(at::kFloat);
  auto mean = torch::empty({R}, fo);
  auto q = torch::empty({R, L}, fo);
  auto srt = return_sorted ? torch::empty({R, K}, fo) : torch::empty({0}, fo);
  if (R == 0) return {mean, q, srt};
  auto s = at::cuda::getCurrentCUDAStream();
  float* so = return_sorted ? srt.data_ptr<float>() : nullptr;
  if (pred.scalar_type() == at::kBFloat16) {
    quantile_decode_kernel<__nv_bfloat16><<<R, 512, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(pred.data_ptr()), R,
                                                             K, taus.data_ptr<float>(), levels.data_ptr<float>(), L,
                                                             mean.data_ptr<float>(), q.data_ptr<float>(), so);
  } else {
    TORCH_CHECK(pred.scalar_type() == at::kFloat, "quantile_decode: bf16 or fp32");
    quantile_decode_kernel<float><<<R, 512, 0, s>>>(pred.data_ptr<float>(), R, K, taus.data_ptr<float>(),
                                                     levels.data_ptr<float>(), L, mean.data_ptr<float>(),
                                                     q.data_ptr<float>(), so);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {mean, q, srt};
}

}  // namespace nori
