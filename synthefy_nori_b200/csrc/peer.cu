// Bucketed data-parallel optimizer step over NVLink / NVSwitch peer memory (no NCCL on
// the path), and the bf16 weight-layout refresh shared with the single-GPU optimizer.
//
// Flat buffers.  Every rank holds the trainable parameters in one fp32 buffer laid out
// in (approximate) backward order and cut into buckets of ~25 MB.  Each bucket is split
// into W pieces (64-element aligned); rank r owns piece r of every bucket: it reduces
// that piece, keeps its AdamW moments and EMA, and updates it.
//
// During the backward pass (comm stream, one bucket at a time, as soon as the bucket's
// last gradient has been accumulated on the compute stream):
//   bucket_pack_signal  casts the bucket's fp32 gradients to the bf16 wire buffer (or
//                       leaves them fp32), then the last CTA to finish publishes
//                       "bucket b ready at step s" into every peer's flag block
//                       (system-scope release);
//   peer_wait           one CTA waits (bounded) until every peer flagged bucket b;
//   bucket_reduce       sums this rank's piece of the bucket over all ranks with P2P
//                       loads, converting bf16 -> fp32 and scaling by 1/W in registers,
//                       and accumulates the piece's sum of squares for the clip.
// After the backward pass:
//   peer_publish        shard norm partial + step status bits (skip / non-finite) to
//                       every peer, then the norm-ready flag;
//   peer_adamw          global clip factor and status from all partials; AdamW + EMA on
//                       the owned pieces only (sharded optimizer state);
//   peer_signal         "params ready";
//   layout_sync         all-gather: every rank reads each peer's updated pieces (plain
//                       P2P loads), writes them into its fp32 master buffer and, in the
//                       same pass, into the bf16 operand layouts the next forward's
//                       GEMMs read (fused QKV / KV rows, interleaved SwiGLU gate/up
//                       rows), so no per-step cast or re-layout of the weights remains.
// Flags hold monotonically increasing step numbers and never need resetting.  All
// peer buffers are cudaMalloc allocations shared once through CUDA IPC handles.  All
// loads from peer memory are plain loads (no TMA, no multicast).  Every wait is bounded
// by a caller-given wall-clock limit; on expiry it records kTimeoutPeer in the device
// status word, and kernels that start after a recorded error return at once.
//
// Reference counterpart: DDP's bucketed NCCL all-reduce with gradient_as_bucket_view
// (training/cli.py:1446-1452), clip_grad_norm_ + AdamW + EMA (training/trainer.py:
// 1544-1552, 38-63), loss-spike skip agreed over ranks (trainer.py:1440-1482).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>

#include "sm100.cuh"
#include "tma_host.h"

namespace nori {

constexpr int kMaxPeers = 8;
constexpr int kMaxBuckets = 1024;

struct PeerSet {
  const void* wire[kMaxPeers];  // gradient wire buffer of each rank (bf16 or fp32, flat)
  float* param[kMaxPeers];      // flat fp32 parameter buffer of each rank
  uint64_t* flags[kMaxPeers];   // flag block of each rank
  float* xchg[kMaxPeers];       // [2W] per rank: shard norm partials, status bits
};

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ bool failed(const int* status) {
  return status != nullptr && *reinterpret_cast<const volatile int*>(status) != 0;
}

// Bounded wait until flags[base + i] >= step for every i < W (the flag block is this
// rank's own memory, written by the peers).  One CTA; lane i polls slot i.
__global__ void peer_wait_kernel(const uint64_t* flags, int base, int W, uint64_t step, uint64_t limit_ns,
                                 int* status) {
  if (threadIdx.x >= W || failed(status)) return;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (ld_acquire_sys(flags + base + threadIdx.x) < step) {
    if ((++spins & 63u) == 0 && globaltimer_ns() - t0 > limit_ns) {
      record_status(status, kTimeoutPeer);
      return;
    }
    __nanosleep(256);
  }
}

// Publish flags[slot + rank] = step into every rank's flag block, after all prior work
// of this stream (system-scope fence, then release stores).
__global__ void peer_signal_kernel(PeerSet ps, int W, int rank, int slot, uint64_t step) {
  __threadfence_system();
  if (threadIdx.x < W) st_release_sys(ps.flags[threadIdx.x] + slot + rank, step);
}

// Cast grad[b0, b0+n) to bf16 into wire (if given), then the last CTA to finish
// publishes bucket-ready.  n and b0 are multiples of 4.
__global__ void bucket_pack_signal_kernel(const float* __restrict__ grad, __nv_bfloat16* __restrict__ wire,
                                          int64_t b0, int64_t n, unsigned* counter, PeerSet ps, int W, int rank,
                                          int slot, uint64_t step) {
  if (wire != nullptr) {
    const int64_t n4 = n / 4;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
      const float4 g = *reinterpret_cast<const float4*>(grad + b0 + 4 * i);
      __nv_bfloat162 lo = __floats2bfloat162_rn(g.x, g.y), hi = __floats2bfloat162_rn(g.z, g.w);
      uint2 pk;
      pk.x = *reinterpret_cast<uint32_t*>(&lo);
      pk.y = *reinterpret_cast<uint32_t*>(&hi);
      *reinterpret_cast<uint2*>(wire + b0 + 4 * i) = pk;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned t = atomicAdd(counter, 1u);
    if (t == gridDim.x - 1) {
      *counter = 0u;  // stream-ordered reuse by the next step
      __threadfence_system();
      for (int p = 0; p < W; ++p) st_release_sys(ps.flags[p] + slot + rank, step);
    }
  }
}

// red[i] = scale * sum_p wire_p[f0 + i] for i < n (n a multiple of 4); norm_acc += sum red^2.
__global__ void bucket_reduce_kernel(PeerSet ps, int W, int64_t f0, int64_t n, int wire_bf16, float scale,
                                     float* __restrict__ red, float* __restrict__ norm_acc, const int* status) {
  if (failed(status)) return;
  float ss = 0.f;
  const int64_t n4 = n / 4;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    const int64_t e = f0 + 4 * i;
    if (wire_bf16) {
#pragma unroll 1
      for (int p = 0; p < W; ++p) {
        const uint2 pk = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(ps.wire[p]) + e);
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&pk.x));
        const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&pk.y));
        acc.x += a.x;
        acc.y += a.y;
        acc.z += b.x;
        acc.w += b.y;
      }
    } else {
#pragma unroll 1
      for (int p = 0; p < W; ++p) {
        const float4 g = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(ps.wire[p]) + e);
        acc.x += g.x;
        acc.y += g.y;
        acc.z += g.z;
        acc.w += g.w;
      }
    }
    acc.x *= scale;
    acc.y *= scale;
    acc.z *= scale;
    acc.w *= scale;
    *reinterpret_cast<float4*>(red + 4 * i) = acc;
    ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
  }
  ss = warp_sum(ss);
  __shared__ float part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? part[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) atomicAdd(norm_acc, v);
  }
}

// xchg_p[rank] = local norm partial, xchg_p[W + rank] = local status bits, for every p;
// then flags_p[slot + rank] = step.
__global__ void peer_publish_kernel(PeerSet ps, int W, int rank, const float* local_norm, const float* local_bits,
                                    int slot, uint64_t step) {
  if (threadIdx.x < W) {
    ps.xchg[threadIdx.x][rank] = *local_norm;
    ps.xchg[threadIdx.x][W + rank] = local_bits != nullptr ? *local_bits : 0.f;
    __threadfence_system();
    st_release_sys(ps.flags[threadIdx.x] + slot + rank, step);
  }
}

struct PeerAdamArgs {
  float lr, beta1, beta2, eps, wd, bc1, bc2_sqrt, ema_decay, max_norm;
  int use_ema;
};

// AdamW + EMA on the owned pieces: piece y = blockIdx.y spans red[tab[3y], +tab[3y+2])
// and param[tab[3y+1], +tab[3y+2]).  The clip factor and the skip decision come from
// the exchanged partials (identical on every rank).  diag (block (0,0)): [0] global
// gradient norm, [1] status bits of the step (> 0: not applied).
__global__ void peer_adamw_kernel(PeerSet ps, int W, int rank, const int64_t* __restrict__ tab,
                                  const float* __restrict__ red, float* __restrict__ m, float* __restrict__ v,
                                  float* __restrict__ ema, PeerAdamArgs a, float* diag, const int* status) {
  if (failed(status)) return;
  __shared__ float scale_s;
  __shared__ int skip_s;
  if (threadIdx.x == 0) {
    const volatile float* x = ps.xchg[rank];
    float tot = 0.f, bits = 0.f;
    for (int p = 0; p < W; ++p) {
      tot += x[p];
      bits = fmaxf(bits, x[W + p]);
    }
    const float norm = sqrtf(tot);
    float scale = 1.f;
    if (a.max_norm > 0.f) {
      const float c = a.max_norm / (norm + 1e-6f);
      if (c < 1.f) scale = c;
    }
    // a non-finite norm (overflowed gradients) skips the step as well
    skip_s = (bits > 0.f || !(norm < INFINITY)) ? 1 : 0;
    scale_s = scale;
    if (blockIdx.x == 0 && blockIdx.y == 0 && diag != nullptr) {
      diag[0] = norm;
      diag[1] = skip_s ? fmaxf(bits, 1.f) : 0.f;
    }
  }
  __syncthreads();
  if (skip_s) return;
  const float scale = scale_s;
  const int64_t roff = tab[3 * blockIdx.y], foff = tab[3 * blockIdx.y + 1], len = tab[3 * blockIdx.y + 2];
  float* param = ps.param[rank] + foff;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < len; i += stride) {
    const int64_t k = roff + i;
    const float gi = red[k] * scale;
    float pi = param[i] * (1.f - a.lr * a.wd);
    const float mi = a.beta1 * m[k] + (1.f - a.beta1) * gi;
    const float vi = a.beta2 * v[k] + (1.f - a.beta2) * gi * gi;
    m[k] = mi;
    v[k] = vi;
    pi -= (a.lr / a.bc1) * mi / (sqrtf(vi) / a.bc2_sqrt + a.eps);
    param[i] = pi;
    if (a.use_ema) ema[k] = a.ema_decay * ema[k] + (1.f - a.ema_decay) * pi;
  }
}

// ------------------------------------------------------------------ layout sync
// Segment table rows (int64 x 5): src flat offset, rows, cols, dst bf16 address (0 = none),
// dst row stride (elements).  Segment element j (row j / cols, column j % cols) is flat
// element src + j.  Chunk table rows (int64 x 3): segment, j0, j1 (multiples of 4).
// Owner of flat element f: bucket b = last b with bstart[b] <= f, piece (f - bstart[b]) /
// bper[b]; with no buckets (single GPU) the owner is this rank.
__global__ void layout_sync_kernel(const int64_t* __restrict__ seg, const int64_t* __restrict__ chunks, int nchunks,
                                   PeerSet ps, int W, int rank, const int64_t* __restrict__ bstart,
                                   const int64_t* __restrict__ bper, int nb, const int* status) {
  __shared__ int64_t s_start[kMaxBuckets + 1];
  __shared__ int64_t s_per[kMaxBuckets];
  if (failed(status)) return;
  for (int i = threadIdx.x; i < nb; i += blockDim.x) {
    s_start[i] = bstart[i];
    s_per[i] = bper[i];
  }
  if (threadIdx.x == 0 && nb > 0) s_start[nb] = bstart[nb];
  __syncthreads();
  float* local = ps.param[rank];
  for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
    const int64_t* ch = chunks + 3 * static_cast<int64_t>(c);
    const int64_t* sg = seg + 5 * ch[0];
    const int64_t src = sg[0], cols = sg[2], dst_rs = sg[4];
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(sg[3]);
    for (int64_t j = ch[1] + 4 * threadIdx.x; j < ch[2]; j += 4 * blockDim.x) {
      const int64_t f = src + j;
      int owner = rank;
      if (nb > 0) {
        int lo = 0, hi = nb - 1;
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (s_start[mid] <= f) lo = mid; else hi = mid - 1;
        }
        owner = static_cast<int>((f - s_start[lo]) / s_per[lo]);
        if (owner >= W) owner = W - 1;
      }
      const float4 val = *reinterpret_cast<const float4*>(ps.param[owner] + f);
      if (owner != rank) *reinterpret_cast<float4*>(local + f) = val;
      if (dst != nullptr) {
        const int64_t r = j / cols, cc = j - r * cols;
        __nv_bfloat162 lo2 = __floats2bfloat162_rn(val.x, val.y), hi2 = __floats2bfloat162_rn(val.z, val.w);
        uint2 pk;
        pk.x = *reinterpret_cast<uint32_t*>(&lo2);
        pk.y = *reinterpret_cast<uint32_t*>(&hi2);
        *reinterpret_cast<uint2*>(dst + r * dst_rs + cc) = pk;
      }
    }
  }
}

// ------------------------------------------------------------------ host
// Pointer set of W ranks; every non-empty list must hold exactly W pointers.
static PeerSet make_set(size_t W, const std::vector<int64_t>& wire, const std::vector<int64_t>& param,
                        const std::vector<int64_t>& flags, const std::vector<int64_t>& xchg) {
  TORCH_CHECK(W >= 1 && W <= static_cast<size_t>(kMaxPeers), "1 to 8 ranks");
  for (const auto* l : {&wire, &param, &flags, &xchg})
    TORCH_CHECK(l->empty() || l->size() == W, "one pointer per rank expected");
  PeerSet ps{};
  for (size_t i = 0; i < W; ++i) {
    ps.wire[i] = wire.empty() ? nullptr : reinterpret_cast<const void*>(wire[i]);
    ps.param[i] = param.empty() ? nullptr : reinterpret_cast<float*>(param[i]);
    ps.flags[i] = flags.empty() ? nullptr : reinterpret_cast<uint64_t*>(flags[i]);
    ps.xchg[i] = xchg.empty() ? nullptr : reinterpret_cast<float*>(xchg[i]);
  }
  return ps;
}

static int* status_ptr(const torch::Tensor& status) {
  TORCH_CHECK(status.is_cuda() && status.scalar_type() == at::kInt && status.numel() >= 1, "status: int32 CUDA word");
  return status.data_ptr<int>();
}

static int sm_count(int dev) {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms > 0 ? sms : 148;
}

void peer_wait(int64_t flags, int64_t base, int64_t W, int64_t step, double limit_s, const torch::Tensor& status) {
  TORCH_CHECK(W >= 1 && W <= kMaxPeers, "peer_wait: 1 to 8 ranks");
  TORCH_CHECK(limit_s > 0.0, "peer_wait: positive wait limit");
  const at::cuda::CUDAGuard guard(status.device());
  const uint64_t ns = static_cast<uint64_t>(limit_s * 1e9);
  peer_wait_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(reinterpret_cast<const uint64_t*>(flags),
                                                                   static_cast<int>(base), static_cast<int>(W),
                                                                   static_cast<uint64_t>(step), ns, status_ptr(status));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void peer_signal(std::vector<int64_t> flags, int64_t rank, int64_t slot, int64_t step) {
  PeerSet ps = make_set(flags.size(), {}, {}, flags, {});
  const int W = static_cast<int>(flags.size());
  peer_signal_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(ps, W, static_cast<int>(rank),
                                                                     static_cast<int>(slot), static_cast<uint64_t>(step));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Pack bucket [b0, b0 + n) of the local gradient (bf16 wire when `wire` != 0) and signal.
void peer_bucket_pack_signal(int64_t grad, int64_t wire, int64_t b0, int64_t n, int64_t counter,
                             std::vector<int64_t> flags, int64_t rank, int64_t slot, int64_t step, int64_t device) {
  TORCH_CHECK(b0 % 4 == 0 && n % 4 == 0 && n >= 0, "bucket bounds must be multiples of 4 elements");
  PeerSet ps = make_set(flags.size(), {}, {}, flags, {});
  const int W = static_cast<int>(flags.size());
  // with SMs reserved for the communication kernels, the pack stays within them
  const int cap = sm_reserve() > 0 ? 2 * sm_reserve() : 2 * sm_count(device);
  const int blocks = wire != 0 ? static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n / 4 + 255) / 256, cap)))
                               : 1;
  bucket_pack_signal_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const float*>(grad), reinterpret_cast<__nv_bfloat16*>(wire), b0, n,
      reinterpret_cast<unsigned*>(counter), ps, W, static_cast<int>(rank), static_cast<int>(slot),
      static_cast<uint64_t>(step));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void peer_bucket_reduce(std::vector<int64_t> wire, int64_t f0, int64_t n, bool wire_bf16, double scale, int64_t red,
                        int64_t norm_acc, const torch::Tensor& status, int64_t ctas) {
  TORCH_CHECK(f0 % 4 == 0 && n % 4 == 0 && n >= 0, "piece bounds must be multiples of 4 elements");
  if (n == 0) return;
  const at::cuda::CUDAGuard guard(status.device());
  PeerSet ps = make_set(wire.size(), wire, {}, {}, {});
  const int W = static_cast<int>(wire.size());
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n / 4 + 255) / 256, ctas)));
  bucket_reduce_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      ps, W, f0, n, wire_bf16 ? 1 : 0, static_cast<float>(scale), reinterpret_cast<float*>(red),
      reinterpret_cast<float*>(norm_acc), status_ptr(status));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void peer_publish(std::vector<int64_t> flags, std::vector<int64_t> xchg, int64_t rank, int64_t local_norm,
                  int64_t local_bits, int64_t slot, int64_t step) {
  TORCH_CHECK(flags.size() == xchg.size(), "peer_publish: one flag block and one exchange buffer per rank");
  PeerSet ps = make_set(flags.size(), {}, {}, flags, xchg);
  const int W = static_cast<int>(flags.size());
  peer_publish_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      ps, W, static_cast<int>(rank), reinterpret_cast<const float*>(local_norm),
      reinterpret_cast<const float*>(local_bits), static_cast<int>(slot), static_cast<uint64_t>(step));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void peer_adamw(std::vector<int64_t> params, std::vector<int64_t> xchg, int64_t rank, const torch::Tensor& tab,
                torch::Tensor& red, torch::Tensor& m, torch::Tensor& v, const c10::optional<torch::Tensor>& ema,
                double lr, double beta1, double beta2, double eps, double wd, int64_t opt_step, double ema_decay,
                double max_norm, int64_t max_piece, const torch::Tensor& diag, const torch::Tensor& status) {
  TORCH_CHECK(tab.is_cuda() && tab.scalar_type() == at::kLong && tab.dim() == 2 && tab.size(1) == 3,
              "peer_adamw: piece table int64 [pieces, 3]");
  TORCH_CHECK(red.scalar_type() == at::kFloat && m.scalar_type() == at::kFloat && v.scalar_type() == at::kFloat,
              "peer_adamw: fp32 shard buffers");
  const at::cuda::CUDAGuard guard(red.device());
  PeerSet ps = make_set(params.size(), {}, params, {}, xchg);
  const int W = static_cast<int>(params.size());
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
  a.use_ema = ema.has_value() && ema->defined() ? 1 : 0;
  const int pieces = static_cast<int>(tab.size(0));
  if (pieces == 0) return;
  TORCH_CHECK(pieces <= 65535, "peer_adamw: too many buckets");
  TORCH_CHECK(diag.is_cuda() && diag.scalar_type() == at::kFloat && diag.numel() >= 2, "peer_adamw: fp32 diag [2]");
  const int gx = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((max_piece + 255) / 256,
                                                                         (4 * sm_count(red.get_device()) + pieces - 1) / pieces)));
  peer_adamw_kernel<<<dim3(gx, pieces), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      ps, W, static_cast<int>(rank), tab.data_ptr<int64_t>(), red.data_ptr<float>(), m.data_ptr<float>(),
      v.data_ptr<float>(), a.use_ema ? ema->data_ptr<float>() : nullptr, a, diag.data_ptr<float>(), status_ptr(status));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// One pass: gather every flat element from its owner (when buckets are given) and
// write the bf16 operand layouts listed in the segment table.
void layout_sync(const torch::Tensor& seg, const torch::Tensor& chunks, std::vector<int64_t> params, int64_t rank,
                 const c10::optional<torch::Tensor>& bstart, const c10::optional<torch::Tensor>& bper,
                 const torch::Tensor& status) {
  TORCH_CHECK(seg.is_cuda() && seg.scalar_type() == at::kLong && seg.dim() == 2 && seg.size(1) == 5,
              "layout_sync: segment table int64 [segments, 5]");
  TORCH_CHECK(chunks.is_cuda() && chunks.scalar_type() == at::kLong && chunks.dim() == 2 && chunks.size(1) == 3,
              "layout_sync: chunk table int64 [chunks, 3]");
  const at::cuda::CUDAGuard guard(seg.device());
  PeerSet ps = make_set(params.size(), {}, params, {}, {});
  const int W = static_cast<int>(params.size());
  TORCH_CHECK(rank >= 0 && rank < W, "layout_sync: rank out of range");
  int nb = 0;
  const int64_t *bs = nullptr, *bp = nullptr;
  if (bstart.has_value() && bstart->defined()) {
    TORCH_CHECK(bper.has_value() && bper->defined(), "layout_sync: bucket starts need piece sizes");
    nb = static_cast<int>(bper->numel());
    TORCH_CHECK(nb <= kMaxBuckets && bstart->numel() == nb + 1, "layout_sync: at most 1024 buckets, starts [nb + 1]");
    bs = bstart->data_ptr<int64_t>();
    bp = bper->data_ptr<int64_t>();
  } else {
    TORCH_CHECK(W == 1, "layout_sync: bucket geometry needed for more than one rank");
  }
  const int nch = static_cast<int>(chunks.size(0));
  if (nch == 0) return;
  const int blocks = std::min(nch, 4 * sm_count(seg.get_device()));
  layout_sync_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      seg.data_ptr<int64_t>(), chunks.data_ptr<int64_t>(), nch, ps, W, static_cast<int>(rank), bs, bp, nb,
      status_ptr(status));
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
