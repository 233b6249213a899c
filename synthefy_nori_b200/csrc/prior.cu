// SCM-prior random-MLP forward for a batch of synthetic tables (K19).
//
// Each table b is a random structural causal model realised as an MLP with its own
// depth, width, activation, weights and noise.  All tables of a step share the row
// count N and are padded to a common width H (columns >= the table's width stay zero),
// so one launch covers the whole batch:
//
//   scm_act     A[b, n, k] = act_b(s_b * ((h[b, n, k] - mu[b, k]) * rstd[b, k] + c_b))
//               (the reference's StdScaleLayer -> RandomScaleLayer -> activation; the
//               column statistics come from the context rows of the previous layer);
//               act_b is one of tanh, leaky-relu, elu, identity, selu, silu, relu,
//               softplus, relu6, hardtanh, sign, exp(-x^2), exp, sqrt|x|, 1{|x|<=1},
//               sin, x^2, |x| or a random-Fourier function sum_f w_f sin(fr_f z + ph_f)
//               of the standardised value (256 frequencies per table and layer);
//   scm_linear  h'[b, n, j] = clamp(sum_k A[b, n, k] W[b, j, k] + bias[b, j]
//                                   + sigma[b, j] * N(0, 1), -100, 100)
//               as a tiled fp32 GEMM (64 x 64 output tile per CTA, 4 x 4 per thread,
//               grid z = table), the Gaussian noise drawn from a counter-based hash of
//               (seed, table, layer, row, column) (SplitMix64 finaliser, Box-Muller),
//               and the fp64 column sums / sums of squares of the context rows
//               accumulated for the next layer's standardisation.
// fp32 throughout (the prior's noise can be as small as 1e-4, below bf16 resolution).
//
// Reference: training/scm_prior_generator.py:58-241 (activations, scale layers),
// 318-338 (Gaussian noise), 402-600 (MLPSCM forward).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "sm100.cuh"

namespace nori {

constexpr int kRff = 256;

enum ScmAct : int {
  kTanh = 0, kLeakyRelu, kElu, kIdentity, kSelu, kSilu, kRelu, kSoftplus, kRelu6, kHardtanh, kSign, kRbf, kExp,
  kSqrtAbs, kUnitInd, kSin, kSquare, kAbs, kRandomFourier, kNumScmActs
};

__device__ __forceinline__ float scm_act_apply(int code, float x) {
  switch (code) {
    case kTanh: return tanhf(x);
    case kLeakyRelu: return x >= 0.f ? x : 0.01f * x;
    case kElu: return x > 0.f ? x : expm1f(x);
    case kIdentity: return x;
    case kSelu: return 1.0507009873554805f * (x > 0.f ? x : 1.6732632423543772f * expm1f(x));
    case kSilu: return x / (1.f + expf(-x));
    case kRelu: return fmaxf(x, 0.f);
    case kSoftplus: return x > 20.f ? x : log1pf(expf(x));
    case kRelu6: return fminf(fmaxf(x, 0.f), 6.f);
    case kHardtanh: return fminf(fmaxf(x, -1.f), 1.f);
    case kSign: return x >= 0.f ? 1.f : -1.f;
    case kRbf: return expf(-x * x);
    case kExp: return expf(x);
    case kSqrtAbs: return sqrtf(fabsf(x));
    case kUnitInd: return fabsf(x) <= 1.f ? 1.f : 0.f;
    case kSin: return sinf(x);
    case kSquare: return x * x;
    case kAbs: return fabsf(x);
    default: return x;
  }
}

// h [B, N, H] -> A [B, N, H].  code / scale / shift [B]; width [B]; mean / rstd [B, H];
// rff [B, 3, 256] (frequency, phase, weight) for tables whose code is RandomFourier.
__global__ void scm_act_kernel(const float* __restrict__ h, int N, int H, const int* __restrict__ code,
                               const float* __restrict__ scale, const float* __restrict__ shift,
                               const int* __restrict__ width, const float* __restrict__ mean,
                               const float* __restrict__ rstd, const float* __restrict__ rff,
                               float* __restrict__ out) {
  const int b = blockIdx.z;
  const int c = code[b];
  const int w = width[b];
  __shared__ float s_rff[3 * kRff];
  if (c == kRandomFourier)
    for (int i = threadIdx.x; i < 3 * kRff; i += blockDim.x) s_rff[i] = rff[static_cast<int64_t>(b) * 3 * kRff + i];
  __syncthreads();
  const float sc = scale[b], sh = shift[b];
  const int64_t total = static_cast<int64_t>(N) * H;
  const float* hb = h + static_cast<int64_t>(b) * total;
  float* ob = out + static_cast<int64_t>(b) * total;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int k = static_cast<int>(i % H);
    if (k >= w) {
      ob[i] = 0.f;
      continue;
    }
    const float z = (hb[i] - mean[static_cast<int64_t>(b) * H + k]) * rstd[static_cast<int64_t>(b) * H + k];
    float v;
    if (c == kRandomFourier) {
      // the random-Fourier activation standardises its (affine) input again, which
      // returns the standardised value z: evaluate the Fourier sum on z
      float acc = 0.f;
#pragma unroll 8
      for (int f = 0; f < kRff; ++f) acc += s_rff[2 * kRff + f] * sinf(s_rff[f] * z + s_rff[kRff + f]);
      v = acc;
    } else {
      v = scm_act_apply(c, sc * (z + sh));
    }
    ob[i] = isfinite(v) ? v : 0.f;
  }
}

// Counter-based standard normal: SplitMix64 finaliser of the counter, two 24-bit
// uniforms, Box-Muller.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__device__ __forceinline__ float gauss(uint64_t seed, uint64_t ctr) {
  const uint64_t r = mix64(seed ^ mix64(ctr));
  const float u1 = (static_cast<float>(r >> 40) + 0.5f) * (1.0f / 16777216.0f);
  const float u2 = static_cast<float>((r >> 16) & 0xFFFFFFull) * (1.0f / 16777216.0f);
  return sqrtf(-2.f * __logf(u1)) * __cosf(6.283185307179586f * u2);
}

constexpr int kTile = 64, kKt = 32;

// out [B, N, Hout] = clamp(A [B, N, K] W[b]^T + bias + noise); W [B, Hout, K]; bias,
// sigma [B, Hout]; out_width [B] (columns beyond are zero); fit_rows rows feed the fp64
// column sums sum / sq [B, Hout] (accumulated).
__global__ void __launch_bounds__(256) scm_linear_kernel(
    const float* __restrict__ A, const float* __restrict__ W, const float* __restrict__ bias,
    const float* __restrict__ sigma, const int* __restrict__ out_width, int N, int K, int Hout, int fit_rows,
    uint64_t seed, int layer, float* __restrict__ out, double* __restrict__ csum, double* __restrict__ csq) {
  const int b = blockIdx.z;
  const int r0 = blockIdx.x * kTile, c0 = blockIdx.y * kTile;
  const int ow = out_width[b];
  if (c0 >= ow) {  // whole tile beyond this table's width: zeros
    for (int i = threadIdx.x; i < kTile * kTile; i += blockDim.x) {
      const int r = r0 + i / kTile, c = c0 + i % kTile;
      if (r < N && c < Hout) out[(static_cast<int64_t>(b) * N + r) * Hout + c] = 0.f;
    }
    return;
  }
  __shared__ float sA[kKt][kTile + 1];
  __shared__ float sW[kKt][kTile + 1];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[4][4] = {};
  const float* Ab = A + static_cast<int64_t>(b) * N * K;
  const float* Wb = W + static_cast<int64_t>(b) * Hout * K;
  for (int k0 = 0; k0 < K; k0 += kKt) {
    for (int i = threadIdx.x; i < kKt * kTile; i += blockDim.x) {
      const int kk = i % kKt, rr = i / kKt;
      const int r = r0 + rr, c = c0 + rr, k = k0 + kk;
      sA[kk][rr] = (r < N && k < K) ? Ab[static_cast<int64_t>(r) * K + k] : 0.f;
      sW[kk][rr] = (c < Hout && k < K) ? Wb[static_cast<int64_t>(c) * K + k] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kKt; ++kk) {
      float a[4], w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = sA[kk][ty * 4 + i];
        w[i] = sW[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], w[j], acc[i][j]);
    }
    __syncthreads();
  }
  // epilogue: bias, noise, clamp, store; context-row column sums via shared memory
  __shared__ float s_sum[16][kTile], s_sq[16][kTile];
  float psum[4] = {0.f, 0.f, 0.f, 0.f}, psq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = r0 + ty * 4 + i;
    if (r >= N) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = c0 + tx * 4 + j;
      if (c >= Hout) continue;
      float v = 0.f;
      if (c < ow) {
        v = acc[i][j] + bias[static_cast<int64_t>(b) * Hout + c];
        const float sg = sigma[static_cast<int64_t>(b) * Hout + c];
        if (sg > 0.f) {
          // (table, layer) in bits 40-61, row in 16-39, column in 0-15
          const uint64_t ctr = ((static_cast<uint64_t>(b) * 64u + static_cast<uint64_t>(layer)) << 40) |
                               (static_cast<uint64_t>(r) << 16) | static_cast<uint64_t>(c);
          v += sg * gauss(seed, ctr);
        }
        v = isfinite(v) ? fminf(fmaxf(v, -100.f), 100.f) : 0.f;
        if (r < fit_rows) {
          psum[j] += v;
          psq[j] += v * v;
        }
      }
      out[(static_cast<int64_t>(b) * N + r) * Hout + c] = v;
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    s_sum[ty][tx * 4 + j] = psum[j];
    s_sq[ty][tx * 4 + j] = psq[j];
  }
  __syncthreads();
  if (threadIdx.x < kTile) {
    const int c = c0 + threadIdx.x;
    if (c < ow && c < Hout) {
      double s = 0.0, q = 0.0;
      for (int t = 0; t < 16; ++t) {
        s += s_sum[t][threadIdx.x];
        q += s_sq[t][threadIdx.x];
      }
      atomicAdd(csum + static_cast<int64_t>(b) * Hout + c, s);
      atomicAdd(csq + static_cast<int64_t>(b) * Hout + c, q);
    }
  }
}

// ------------------------------------------------------------------ host
static void c32(const torch::Tensor& t, at::ScalarType dt, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == dt && t.is_contiguous(), what, ": contiguous CUDA tensor of the right dtype");
}

torch::Tensor scm_act(const torch::Tensor& h, const torch::Tensor& code, const torch::Tensor& scale,
                      const torch::Tensor& shift, const torch::Tensor& width, const torch::Tensor& mean,
                      const torch::Tensor& rstd, const torch::Tensor& rff) {
  c32(h, at::kFloat, "h");
  TORCH_CHECK(h.dim() == 3, "scm_act: h [B, N, H]");
  const int B = static_cast<int>(h.size(0)), N = static_cast<int>(h.size(1)), H = static_cast<int>(h.size(2));
  c32(code, at::kInt, "code");
  c32(width, at::kInt, "width");
  c32(scale, at::kFloat, "scale");
  c32(shift, at::kFloat, "shift");
  c32(mean, at::kFloat, "mean");
  c32(rstd, at::kFloat, "rstd");
  c32(rff, at::kFloat, "rff");
  TORCH_CHECK(code.numel() == B && width.numel() == B && scale.numel() == B && shift.numel() == B,
              "scm_act: one code / width / scale / shift per table");
  TORCH_CHECK(mean.numel() == static_cast<int64_t>(B) * H && rstd.numel() == mean.numel(), "scm_act: stats [B, H]");
  TORCH_CHECK(rff.numel() == static_cast<int64_t>(B) * 3 * kRff, "scm_act: rff [B, 3, 256]");
  const at::cuda::CUDAGuard guard(h.device());
  auto out = torch::empty_like(h);
  const int64_t per = static_cast<int64_t>(N) * H;
  if (per == 0 || B == 0) return out;
  const dim3 grid(static_cast<unsigned>(std::min<int64_t>((per + 255) / 256, 1024)), 1, B);
  scm_act_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      h.data_ptr<float>(), N, H, code.data_ptr<int>(), scale.data_ptr<float>(), shift.data_ptr<float>(),
      width.data_ptr<int>(), mean.data_ptr<float>(), rstd.data_ptr<float>(), rff.data_ptr<float>(),
      out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

// Returns out [B, N, Hout]; adds context-row column sums / squares into csum / csq (fp64 [B, Hout]).
torch::Tensor scm_linear(const torch::Tensor& A, const torch::Tensor& W, const torch::Tensor& bias,
                         const torch::Tensor& sigma, const torch::Tensor& out_width, int64_t fit_rows, int64_t seed,
                         int64_t layer, torch::Tensor& csum, torch::Tensor& csq) {
  c32(A, at::kFloat, "A");
  c32(W, at::kFloat, "W");
  TORCH_CHECK(A.dim() == 3 && W.dim() == 3 && W.size(0) == A.size(0) && W.size(2) == A.size(2),
              "scm_linear: A [B, N, K], W [B, Hout, K]");
  const int B = static_cast<int>(A.size(0)), N = static_cast<int>(A.size(1)), K = static_cast<int>(A.size(2));
  const int Hout = static_cast<int>(W.size(1));
  c32(bias, at::kFloat, "bias");
  c32(sigma, at::kFloat, "sigma");
  c32(out_width, at::kInt, "out_width");
  c32(csum, at::kDouble, "csum");
  c32(csq, at::kDouble, "csq");
  TORCH_CHECK(bias.numel() == static_cast<int64_t>(B) * Hout && sigma.numel() == bias.numel() &&
                  csum.numel() == bias.numel() && csq.numel() == bias.numel() && out_width.numel() == B,
              "scm_linear: per-table [B, Hout] vectors");
  TORCH_CHECK(layer >= 0 && layer < 64, "scm_linear: layer index < 64");
  TORCH_CHECK(N < (1 << 24) && Hout < 65536 && B < 65536, "scm_linear: N < 2^24, Hout < 65536, B < 65536");
  const at::cuda::CUDAGuard guard(A.device());
  auto out = torch::empty({B, N, Hout}, A.options());
  if (B == 0 || N == 0 || Hout == 0) return out;
  const dim3 grid((N + kTile - 1) / kTile, (Hout + kTile - 1) / kTile, B);
  TORCH_CHECK(grid.x < 2147483647u && grid.y < 65536u && grid.z < 65536u, "scm_linear: grid too large");
  scm_linear_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      A.data_ptr<float>(), W.data_ptr<float>(), bias.data_ptr<float>(), sigma.data_ptr<float>(),
      out_width.data_ptr<int>(), N, K, Hout, static_cast<int>(fit_rows), static_cast<uint64_t>(seed),
      static_cast<int>(layer), out.data_ptr<float>(), csum.data_ptr<double>(), csq.data_ptr<double>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

}  // namespace nori
