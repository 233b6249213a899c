// Peer-memory data-parallel optimizer step over NVLink / NVSwitch (no NCCL on the path).
//
// Every rank owns one contiguous shard of the flat fp32 parameter / gradient buffers.
// After the backward pass:
//   1. peer_signal       each rank stores `step` into slot [rank] of every peer's flag
//                        array (system-scope release; grads are complete in stream order);
//   2. peer_reduce_norm  waits (bounded) for all ranks' flags, sums its shard of the
//                        gradient over all ranks with P2P loads, keeps the reduced shard
//                        locally, and publishes the shard's sum of squares to every peer;
//   3. peer_adamw        waits for all norm partials, derives the global clip factor,
//                        applies AdamW + EMA to the owned shard only (the optimizer state
//                        m / v / ema is sharded: 1 / world of the memory), writes the new
//                        master shard and publishes "params ready";
//   4. peer_allgather    waits for every peer's "params ready" and copies the peers'
//                        updated shards into the local full parameter buffer (P2P loads).
// Flags hold monotonically increasing step numbers, so they never need resetting. Each
// peer buffer is a cudaMalloc'ed allocation shared by CUDA IPC handles exchanged once at
// start-up. All loads from peer memory are plain loads (no TMA, no multicast).
//
// Reference counterpart: DDP's bucketed NCCL all-reduce (training/cli.py:1446-1452),
// clip_grad_norm_ + AdamW + EMA (training/trainer.py:1544-1552, 38-63).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "sm100.cuh"

namespace nori {

constexpr int kMaxPeers = 8;
constexpr uint64_t kPeerWaitNs = 60ull * 1000000000ull;  // 60 s: ranks may legitimately drift

struct PeerPtrs {
  float* grad[kMaxPeers];        // full flat gradient buffer of each rank
  float* param[kMaxPeers];       // full flat fp32 parameter buffer of each rank
  uint64_t* flags[kMaxPeers];    // per-rank flag block: [0, W) ready, [W, 2W) norm-ready, [2W, 3W) params-ready
  float* norms[kMaxPeers];       // per-rank [W] shard norm partials
};

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Wait until flags[base + i] >= step for all i < W (local memory, written by peers).
__device__ bool wait_flags(const uint64_t* flags, int base, int W, uint64_t step, int* status) {
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    ok_s = 1;
    const uint64_t t0 = globaltimer_ns();
    for (int i = 0; i < W; ++i) {
      uint32_t spins = 0;
      while (ld_acquire_sys(flags + base + i) < step) {
        if ((++spins & 1023u) == 0 && globaltimer_ns() - t0 > kPeerWaitNs) {
          record_status(status, kTimeoutPeer);
          ok_s = 0;
          break;
        }
        __nanosleep(200);
      }
      if (!ok_s) break;
    }
  }
  __syncthreads();
  return ok_s != 0;
}

__global__ void peer_signal_kernel(PeerPtrs pp, int W, int rank, int base, uint64_t step) {
  // all prior work of this stream is complete when this kernel runs; make it visible
  __threadfence_system();
  if (threadIdx.x < W) st_release_sys(pp.flags[threadIdx.x] + base + rank, step);
}

// reduce shard [s0, s1) of the gradient over all ranks into `red` (local), norm partial.
__global__ void peer_reduce_norm_kernel(PeerPtrs pp, int W, int rank, int64_t s0, int64_t s1, uint64_t step,
                                        float* __restrict__ red, float* __restrict__ local_norm, int* status) {
  if (!wait_flags(pp.flags[rank], 0, W, step, status)) return;
  float ss = 0.f;
  const int64_t n = s1 - s0;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i * 4 < n; i += stride) {
    const int64_t e = s0 + i * 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (e + 3 < s1) {
#pragma unroll 1
      for (int p = 0; p < W; ++p) {
        const float4 g = *reinterpret_cast<const float4*>(pp.grad[p] + e);
        acc.x += g.x;
        acc.y += g.y;
        acc.z += g.z;
        acc.w += g.w;
      }
      *reinterpret_cast<float4*>(red + (e - s0)) = acc;
      ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
    } else {
      for (int64_t k = e; k < s1; ++k) {
        float a = 0.f;
        for (int p = 0; p < W; ++p) a += pp.grad[p][k];
        red[k - s0] = a;
        ss += a * a;
      }
    }
  }
  ss = warp_sum(ss);
  __shared__ float part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? part[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) atomicAdd(local_norm, v);
  }
}

// publish the local shard norm to every peer's norms[rank], then the norm-ready flag
__global__ void peer_publish_norm_kernel(PeerPtrs pp, int W, int rank, const float* local_norm, uint64_t step) {
  if (threadIdx.x < W) {
    pp.norms[threadIdx.x][rank] = *local_norm;
    __threadfence_system();
    st_release_sys(pp.flags[threadIdx.x] + W + rank, step);
  }
}

struct PeerAdamArgs {
  float lr, beta1, beta2, eps, wd, bc1, bc2_sqrt, ema_decay, max_norm, grad_scale;
  int use_ema;
};

__global__ void peer_adamw_kernel(PeerPtrs pp, int W, int rank, int64_t s0, int64_t s1, uint64_t step,
                                  const float* __restrict__ red, float* __restrict__ m, float* __restrict__ v,
                                  float* __restrict__ ema, PeerAdamArgs a, int* status) {
  if (!wait_flags(pp.flags[rank], W, W, step, status)) return;
  __shared__ float scale_s;
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int p = 0; p < W; ++p) tot += reinterpret_cast<volatile float*>(pp.norms[rank])[p];
    float scale = a.grad_scale;
    if (a.max_norm > 0.f) {
      const float norm = sqrtf(tot) * a.grad_scale;
      const float c = a.max_norm / (norm + 1e-6f);
      if (c < 1.f) scale *= c;
    }
    scale_s = scale;
  }
  __syncthreads();
  const float scale = scale_s;
  float* param = pp.param[rank];
  const int64_t n = s1 - s0;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float gi = red[i] * scale;
    float pi = param[s0 + i] * (1.f - a.lr * a.wd);
    const float mi = a.beta1 * m[i] + (1.f - a.beta1) * gi;
    const float vi = a.beta2 * v[i] + (1.f - a.beta2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    pi -= (a.lr / a.bc1) * mi / (sqrtf(vi) / a.bc2_sqrt + a.eps);
    param[s0 + i] = pi;
    if (a.use_ema) ema[i] = a.ema_decay * ema[i] + (1.f - a.ema_decay) * pi;
  }
}

// copy every peer's updated shard into the local parameter buffer
__global__ void peer_allgather_kernel(PeerPtrs pp, int W, int rank, const int64_t* __restrict__ bounds,
                                      uint64_t step, int* status) {
  if (!wait_flags(pp.flags[rank], 2 * W, W, step, status)) return;
  float* dst = pp.param[rank];
  for (int p = 0; p < W; ++p) {
    if (p == rank) continue;
    const int64_t b0 = bounds[p], b1 = bounds[p + 1];
    const float* src = pp.param[p];
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = b0 + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < b1; i += stride)
      dst[i] = src[i];
  }
}

// ------------------------------------------------------------------ host
static PeerPtrs to_ptrs(const std::vector<int64_t>& grads, const std::vector<int64_t>& params,
                        const std::vector<int64_t>& flags, const std::vector<int64_t>& norms) {
  PeerPtrs pp{};
  TORCH_CHECK(grads.size() <= static_cast<size_t>(kMaxPeers), "at most 8 ranks");
  for (size_t i = 0; i < grads.size(); ++i) {
    pp.grad[i] = reinterpret_cast<float*>(grads[i]);
    pp.param[i] = reinterpret_cast<float*>(params[i]);
    pp.flags[i] = reinterpret_cast<uint64_t*>(flags[i]);
    pp.norms[i] = reinterpret_cast<float*>(norms[i]);
  }
  return pp;
}

// One complete data-parallel optimizer step (four launches on the current stream).
void peer_ddp_step(std::vector<int64_t> grads, std::vector<int64_t> params, std::vector<int64_t> flags,
                   std::vector<int64_t> norms, int64_t rank, int64_t s0, int64_t s1, const torch::Tensor& bounds,
                   int64_t step,
                   torch::Tensor& red, torch::Tensor& m, torch::Tensor& v, const c10::optional<torch::Tensor>& ema,
                   torch::Tensor& local_norm, double lr, double beta1, double beta2, double eps, double wd,
                   int64_t opt_step, double ema_decay, double max_norm, double grad_scale, const torch::Tensor& status) {
  const int W = static_cast<int>(grads.size());
  TORCH_CHECK(W >= 1 && params.size() == grads.size() && flags.size() == grads.size() && norms.size() == grads.size(),
              "peer_ddp_step: one pointer per rank");
  TORCH_CHECK(bounds.scalar_type() == at::kLong && bounds.is_cuda() && bounds.numel() == W + 1, "bounds: int64 [W+1]");
  const at::cuda::CUDAGuard guard(red.device());
  TORCH_CHECK(s0 % 4 == 0 && s1 >= s0, "shard starts must be 16-byte aligned");
  TORCH_CHECK(red.numel() >= s1 - s0 && m.numel() >= s1 - s0 && v.numel() >= s1 - s0, "shard buffers too small");
  PeerPtrs pp = to_ptrs(grads, params, flags, norms);
  auto stream = at::cuda::getCurrentCUDAStream();
  int* st = status.data_ptr<int>();
  const uint64_t sv = static_cast<uint64_t>(step);
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, red.get_device());
  peer_signal_kernel<<<1, 32, 0, stream>>>(pp, W, static_cast<int>(rank), 0, sv);
  local_norm.zero_();
  peer_reduce_norm_kernel<<<sms * 2, 512, 0, stream>>>(pp, W, static_cast<int>(rank), s0, s1, sv,
                                                       red.data_ptr<float>(), local_norm.data_ptr<float>(), st);
  peer_publish_norm_kernel<<<1, 32, 0, stream>>>(pp, W, static_cast<int>(rank), local_norm.data_ptr<float>(), sv);
  PeerAdamArgs a;
  a.lr = static_cast<float>(lr);
  a.beta1 = static_cast<float>(beta1);
  a.beta2 = static_cast<float>(beta2);
  a.eps = static_cast<float>(eps);
  a.wd = static_cast<float>(wd);
  a.bc1 = static_cast<float>(1.0 - std::pow(beta1, static_cast<double>(opt_step)));
  a.bc2_sqrt = static_cast<float>(std::sqrt(1.0 - std::pow(beta2, static_cast<double>(opt_step))));
  a.ema_decay = static_cast<float>(ema_decay);
  a.max_norm = static_cast<float>(max_norm);
  a.grad_scale = static_cast<float>(grad_scale);
  a.use_ema = ema.has_value() && ema->defined() ? 1 : 0;
  peer_adamw_kernel<<<sms * 2, 512, 0, stream>>>(pp, W, static_cast<int>(rank), s0, s1, sv, red.data_ptr<float>(),
                                                 m.data_ptr<float>(), v.data_ptr<float>(),
                                                 a.use_ema ? ema->data_ptr<float>() : nullptr, a, st);
  peer_signal_kernel<<<1, 32, 0, stream>>>(pp, W, static_cast<int>(rank), 2 * W, sv);
  peer_allgather_kernel<<<sms * 2, 512, 0, stream>>>(pp, W, static_cast<int>(rank), bounds.data_ptr<int64_t>(), sv, st);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ---- IPC buffers: raw cudaMalloc allocations (IPC-shareable), wrapped as tensors
int64_t peer_malloc(int64_t bytes) {
  void* p = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&p, static_cast<size_t>(bytes)));
  C10_CUDA_CHECK(cudaMemset(p, 0, static_cast<size_t>(bytes)));
  return reinterpret_cast<int64_t>(p);
}

void peer_free(int64_t ptr) { C10_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr))); }

torch::Tensor peer_ipc_handle(int64_t ptr) {
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(ptr)));
  auto t = torch::empty({static_cast<int64_t>(sizeof(h))}, torch::kUInt8);
  std::memcpy(t.data_ptr(), &h, sizeof(h));
  return t;
}

int64_t peer_ipc_open(const torch::Tensor& handle) {
  TORCH_CHECK(handle.numel() == static_cast<int64_t>(sizeof(cudaIpcMemHandle_t)), "bad IPC handle");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.contiguous().data_ptr(), sizeof(h));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void peer_ipc_close(int64_t ptr) { C10_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr))); }

torch::Tensor tensor_from_ptr(int64_t ptr, int64_t numel, int64_t device, c10::ScalarType dtype) {
  auto opts = torch::TensorOptions().dtype(dtype).device(torch::kCUDA, static_cast<int>(device));
  return torch::from_blob(reinterpret_cast<void*>(ptr), {numel}, [](void*) {}, opts);
}

}  // namespace nori
