// Per-head RMS normalisation with a learned gain, in place, for the two-phase (Model v3,
// nori-1-5) encoder's attention: every attention there normalises its queries and keys per
// head (RMSNorm over the head dimension, eps 1e-6, learned gain) and the queries are then
// multiplied by log(key count) (reference model/two_phase.py:34-50, model/layer.py:497-503,
// 606-630, 440-448). The projection GEMM writes the heads as adjacent D-wide column blocks
// of a bf16 row; this kernel rescales each block where it lies.
//
// Work split: eight lanes per (row, head), each lane owning 8 consecutive bf16 (one 16-byte
// vector), so one warp covers four heads and D <= 64 needs no second pass; the sum of
// squares is reduced over the eight lanes with xor shuffles. fp32 arithmetic, one bf16
// rounding on the way out.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>

namespace nori {
namespace {

__global__ void head_rmsnorm_kernel(__nv_bfloat16* __restrict__ x, int64_t rows, int64_t ld, int heads, int D,
                                    const float* __restrict__ gain, float eps, float post) {
  const int64_t slot = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 3;  // (row, head)
  const int sub = threadIdx.x & 7;
  const int64_t row = slot / heads;
  const int h = static_cast<int>(slot % heads);
  const bool live = row < rows;
  const int c0 = sub * 8;
  const bool mine = live && c0 < D;
  __nv_bfloat16* p = x + (live ? row * ld + static_cast<int64_t>(h) * D + c0 : 0);
  float v[8];
  float ss = 0.f;
  if (mine) {
    const uint4 raw = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h2[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
      ss += f.x * f.x + f.y * f.y;
    }
  }
  // the eight lanes of one (row, head) are aligned within the warp
  ss += __shfl_xor_sync(0xffffffffu, ss, 4);
  ss += __shfl_xor_sync(0xffffffffu, ss, 2);
  ss += __shfl_xor_sync(0xffffffffu, ss, 1);
  if (!mine) return;
  const float r = rsqrtf(ss / static_cast<float>(D) + eps) * post;
  uint4 out;
  __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float g0 = gain ? gain[c0 + 2 * i] : 1.f;
    const float g1 = gain ? gain[c0 + 2 * i + 1] : 1.f;
    o2[i] = __floats2bfloat162_rn(v[2 * i] * r * g0, v[2 * i + 1] * r * g1);
  }
  *reinterpret_cast<uint4*>(p) = out;
}

}  // namespace

// x: bf16 [rows, >= heads * D] with row stride ld (elements); each D-wide head block is
// replaced by rms_normalise(block) * gain * post. gain: fp32 [D] or None.
void head_rmsnorm_(torch::Tensor& x, int64_t heads, int64_t D, const c10::optional<torch::Tensor>& gain, double eps,
                   double post) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2, "head_rmsnorm_: bf16 CUDA matrix");
  TORCH_CHECK(x.stride(1) == 1, "head_rmsnorm_: unit column stride");
  TORCH_CHECK(D > 0 && D <= 64 && D % 8 == 0, "head_rmsnorm_: head dim a multiple of 8, at most 64");
  TORCH_CHECK(heads > 0 && heads * D <= x.size(1), "head_rmsnorm_: heads * D exceeds the row");
  TORCH_CHECK(x.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
              "head_rmsnorm_: 16-byte aligned rows");
  const float* g = nullptr;
  if (gain.has_value() && gain->defined()) {
    TORCH_CHECK(gain->is_cuda() && gain->scalar_type() == at::kFloat && gain->numel() == D && gain->is_contiguous(),
                "head_rmsnorm_: fp32 gain [D]");
    g = gain->data_ptr<float>();
  }
  const at::cuda::CUDAGuard guard(x.device());
  const int64_t rows = x.size(0);
  if (rows == 0) return;
  const int64_t threads = rows * heads * 8;
  constexpr int kBlock = 256;
  const int64_t blocks = (threads + kBlock - 1) / kBlock;
  TORCH_CHECK(blocks < 2147483647LL, "head_rmsnorm_: too many rows");
  head_rmsnorm_kernel<<<static_cast<unsigned>(blocks), kBlock, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), rows, x.stride(0), static_cast<int>(heads),
      static_cast<int>(D), g, static_cast<float>(eps), static_cast<float>(post));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace nori
