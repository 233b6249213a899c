// Feature (within-row) attention on the 5th-generation tensor cores for table rows of at
// most 64 tokens (reference model/layer.py:1391-1405: per table row and head, the G + 1
// tokens of the row attend to each other).
//
// Work item = (two table rows, one head). The 128 MMA lanes hold the two rows' tokens in
// two halves of 64 token slots (row 2p in lanes 0..63, row 2p + 1 in lanes 64..127), and
// the key axis is laid out the same way, so one M=128 x N=128 score MMA computes both
// rows' score blocks on the diagonal; the off-diagonal blocks are never read, and P is
// written back with zeros there, so P . V over all 128 keys only sums each row's own
// keys. Every Q / K / V tile is two TMA boxes of 64 token slots x 64 dims read straight
// from the token-major projection output through a 5-D tensor map whose token extent is
// the row length T and whose column extent is the head width: slots past T and columns
// past the head width arrive as zeros.
//
// Persistent, one CTA per SM, 320 threads:
//   warp 0      TMA producer: Q / K / V of an item (6 boxes, 48 KB) into a 4-stage ring;
//   warp 1      TMEM owner + MMA issuer: S_i = Q K^T (M=128, N=128, K=64) into score buffer
//               i % 2, then O_i = P_i V (M=128, N=64, K=128; A = P_i from TMEM, V read
//               MN-major) into accumulator i % 2, in the order S_0, S_1, PV_0, S_2, PV_1, ...
//   warps 2..5 / 6..9  two softmax + epilogue groups taking alternate items (group g owns
//               score buffer g and accumulator g), thread = MMA lane = token slot: the 64
//               score columns of its own row block, exact max, P (bf16 pairs) over the first
//               64 columns of the score buffer; then the group's previous item's O / l to
//               global memory and its LSE.
// Every mbarrier wait is bounded (sm100.cuh); on timeout the CTA records an error in the
// status word and returns after freeing its TMEM.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <algorithm>

#include "sm100.cuh"
#include "tma_host.h"

namespace nori {

// 2^x as one MUFU instruction (ex2.approx.ftz: flushes subnormal results to zero, which the bf16
// probabilities cannot hold anyway; the arguments are <= 0 after the LSE subtraction). Used by the
// backward's P recomputation (2.94 -> 2.84 ms at 19200 rows x 51 tokens); the forward measured
// no gain from it and keeps exp2f.
__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

namespace ff {
constexpr int kSlots = 64;            // token slots per table row (one half of the MMA lanes)
constexpr int kD = 64;                // padded head dim
constexpr int kThreads = 320;         // warps 0 (TMA), 1 (MMA), 2..9 (two softmax / epilogue groups)
constexpr int kBox = kSlots * kD * 2;  // 8 KB: one row's token slots of one head
constexpr int kTile = 2 * kBox;        // 16 KB: Q, K or V of an item
constexpr int kStages = 4;
constexpr int kSmemBytes = kStages * 3 * kTile + 1024 + 256;
constexpr uint32_t kTmemCols = 512;  // S / P [2] x 128 at 0, 128; O [2] x 64 at 256, 320
}  // namespace ff

struct FeatTcParams {
  int T;        // tokens per table row (<= 64)
  int d_valid;  // head width (multiple of 8, <= 64)
  int H;        // heads
  int64_t n_rows;   // table rows
  int64_t n_items;  // ceil(n_rows / 2) * H
  float scale_log2;
  int q_pos[4], kv_pos[4];  // positions of (token, head, -, table row) inside the 5-D maps
  __nv_bfloat16* o;
  int64_t o_s0, o_s2, o_row;  // output strides of table row, head, token
  float* lse;                 // [n_rows * H, T] natural-log LSE (bh = row * H + head), or null
  int* status;
};

namespace {
__device__ __forceinline__ void feat_coords(const int (&pos)[4], int head, int64_t row, int (&c)[5]) {
  c[0] = 0;
  c[pos[0]] = 0;
  c[pos[1]] = head;
  c[pos[2]] = 0;
  c[pos[3]] = static_cast<int>(row);
}
}  // namespace

__global__ void __launch_bounds__(ff::kThreads, 1)
    attn_feat_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, FeatTcParams p) {
  using namespace ff;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // stage s: Q | K | V, 16 KB each
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * 3 * kTile);
  uint64_t* kv_full = bars;               // [kStages]
  uint64_t* kv_empty = bars + kStages;    // [kStages]
  uint64_t* s_full = bars + 2 * kStages;  // [2]
  uint64_t* p_full = s_full + 2;          // [2]
  uint64_t* o_full = s_full + 4;          // [2]
  uint64_t* o_free = s_full + 6;          // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_full + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t n_items = p.n_items;
  if (p.status != nullptr && *reinterpret_cast<volatile int*>(p.status) != 0) return;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);  // the four warps of group i
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + 256;

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      int it = 0;
      for (int64_t w = blockIdx.x; w < n_items; w += gridDim.x, ++it) {
        const int st = it % kStages;
        if (!mbar_wait(&kv_empty[st], ((it / kStages) & 1) ^ 1, p.status, kTimeoutProducer, abort_flag)) break;
        const int head = static_cast<int>(w % p.H);
        const int64_t row0 = (w / p.H) * 2;
        uint8_t* dst = smem + st * 3 * kTile;
        mbar_arrive_expect_tx(&kv_full[st], 3 * kTile);
        int c[5];
        for (int half = 0; half < 2; ++half) {
          feat_coords(p.q_pos, head, row0 + half, c);
          tma_load_5d(dst + half * kBox, &tmQ, &kv_full[st], c);
          feat_coords(p.kv_pos, head, row0 + half, c);
          tma_load_5d(dst + kTile + half * kBox, &tmK, &kv_full[st], c);
          tma_load_5d(dst + 2 * kTile + half * kBox, &tmV, &kv_full[st], c);
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(128, 128, false, false);
      constexpr uint32_t idesc_o = umma_idesc_bf16(128, kD, false, true);
      bool ok = true;
      // O_i = P_i V_i for the item issued one step earlier
      auto issue_pv = [&](int i) -> bool {
        const int b = i & 1, st = i % kStages;
        if (!mbar_wait(&p_full[b], (i >> 1) & 1, p.status, kTimeoutMma, abort_flag)) return false;
        if (i >= 2 && !mbar_wait(&o_free[b], ((i >> 1) - 1) & 1, p.status, kTimeoutMma, abort_flag)) return false;
        tc_fence_after();
        const uint32_t bV = smem_u32(smem + st * 3 * kTile + 2 * kTile);
#pragma unroll
        for (int k = 0; k < 128 / 16; ++k)
          umma_bf16_ts(tO + b * kD, tS + b * 128 + k * 8, umma_smem_desc(bV + k * 2048, 8192, 1024, 2), idesc_o,
                       k > 0 ? 1u : 0u);
        umma_commit(&o_full[b]);
        umma_commit(&kv_empty[st]);
        return true;
      };
      int it = 0;
      for (int64_t w = blockIdx.x; ok && w < n_items; w += gridDim.x, ++it) {
        const int st = it % kStages, b = it & 1;
        if (!(ok = mbar_wait(&kv_full[st], (it / kStages) & 1, p.status, kTimeoutMma, abort_flag))) break;
        tc_fence_after();
        // S_i goes into the buffer P_{i-2} occupied; PV_{i-2} was issued before this MMA and
        // tcgen05.mma of one thread execute in issue order
        const uint32_t aQ = smem_u32(smem + st * 3 * kTile), bK = aQ + kTile;
#pragma unroll
        for (int k = 0; k < kD / 16; ++k)
          umma_bf16_ss(tS + b * 128, umma_desc_kmajor_sw128(aQ + k * 32), umma_desc_kmajor_sw128(bK + k * 32),
                       idesc_s, k > 0 ? 1u : 0u);
        umma_commit(&s_full[b]);
        if (it >= 1) ok = issue_pv(it - 1);
      }
      if (ok && it >= 1) issue_pv(it - 1);
    }
  } else {
    // ------------------------------------------------------------ softmax / epilogue
    const int q4 = warp & 3;           // TMEM lane quarter this warp may access
    const int r = q4 * 32 + lane;      // MMA lane
    const int half = r >> 6;           // which table row of the item
    const int slot = r & 63;           // token slot inside the row
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    const int T = p.T;
    bool ok = true;
    float prev_m = 0.f, prev_l = 0.f;
    int64_t prev_w = -1;
    auto epilogue = [&](int i, int64_t w, float m, float l) -> bool {
      const int b = i & 1;
      if (!mbar_wait_warp(&o_full[b], (i >> 1) & 1, p.status, kTimeoutEpilogue, abort_flag)) return false;
      tc_fence_after();
      uint32_t oa[32], ob[32];
      tmem_ld32(tO + b * kD + lane_off, oa);
      tmem_ld32(tO + b * kD + 32 + lane_off, ob);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free[b]);
      const int head = static_cast<int>(w % p.H);
      const int64_t row = (w / p.H) * 2 + half;
      if (slot < T && row < p.n_rows) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
        __nv_bfloat16* out = p.o + row * p.o_s0 + static_cast<int64_t>(head) * p.o_s2 + slot * p.o_row;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          if (c8 * 8 >= p.d_valid) break;
          const uint32_t* src = c8 < 4 ? oa + c8 * 8 : ob + (c8 - 4) * 8;
          *reinterpret_cast<uint4*>(out + c8 * 8) =
              make_uint4(pack_bf16x2(__uint_as_float(src[0]) * inv, __uint_as_float(src[1]) * inv),
                         pack_bf16x2(__uint_as_float(src[2]) * inv, __uint_as_float(src[3]) * inv),
                         pack_bf16x2(__uint_as_float(src[4]) * inv, __uint_as_float(src[5]) * inv),
                         pack_bf16x2(__uint_as_float(src[6]) * inv, __uint_as_float(src[7]) * inv));
        }
        if (p.lse != nullptr) {
          constexpr float kLn2 = 0.6931471805599453f;
          p.lse[(row * p.H + head) * T + slot] = l > 0.f ? (m + log2f(l)) * kLn2 : -INFINITY;
        }
      }
      return true;
    };
    const int grp = (warp - 2) >> 2;  // items it with it % 2 == grp
    int it = grp;
    for (int64_t w = blockIdx.x + static_cast<int64_t>(grp) * gridDim.x; ok && w < n_items;
         w += 2 * static_cast<int64_t>(gridDim.x), it += 2) {
      const int b = grp;
      if (!(ok = mbar_wait_warp(&s_full[b], (it >> 1) & 1, p.status, kTimeoutEpilogue, abort_flag))) break;
      tc_fence_after();
      uint32_t sa[32], sb[32];
      const uint32_t tSb = tS + b * 128 + lane_off;
      tmem_ld32(tSb + half * 64, sa);
      tmem_ld32(tSb + half * 64 + 32, sb);
      tmem_wait_ld();
      // scores of this row's keys (slots < T); the rest of the 128 columns is never read
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (j < T) mx = fmaxf(mx, __uint_as_float(sa[j]));
        if (32 + j < T) mx = fmaxf(mx, __uint_as_float(sb[j]));
      }
      const float ms = mx * p.scale_log2;
      float l = 0.f;
      uint32_t pk[32];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float e0 = 2 * j < T ? exp2f(fmaf(__uint_as_float(sa[2 * j]), p.scale_log2, -ms)) : 0.f;
        const float e1 = 2 * j + 1 < T ? exp2f(fmaf(__uint_as_float(sa[2 * j + 1]), p.scale_log2, -ms)) : 0.f;
        const float e2 = 32 + 2 * j < T ? exp2f(fmaf(__uint_as_float(sb[2 * j]), p.scale_log2, -ms)) : 0.f;
        const float e3 = 33 + 2 * j < T ? exp2f(fmaf(__uint_as_float(sb[2 * j + 1]), p.scale_log2, -ms)) : 0.f;
        l += (e0 + e1) + (e2 + e3);
        pk[j] = pack_bf16x2(e0, e1);
        pk[16 + j] = pack_bf16x2(e2, e3);
      }
      // P over the first 64 columns of the score buffer: this row's keys in the columns of
      // its half, zeros in the other half's columns
      uint32_t zero[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) zero[j] = 0u;
      tmem_st32(tSb + half * 32, pk);
      tmem_st32(tSb + (half ^ 1) * 32, zero);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[b]);
      if (it >= 2 && !(ok = epilogue(it - 2, prev_w, prev_m, prev_l))) break;
      prev_w = w;
      prev_m = ms;
      prev_l = l;
    }
    if (ok && it >= 2) epilogue(it - 2, prev_w, prev_m, prev_l);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, ff::kTmemCols);
  }
}

// ------------------------------------------------------------------ backward
// Same item pairing; thread = MMA lane = query slot for S, dP, dQ and = key slot for dK,
// dV (the two run over the same token slots). Per item:
//   S  = Q K^T   (M=128 q, N=128 keys, K=64)  -> TMEM 0..127
//   dP = dO V^T  (M=128 q, N=128 keys, K=64)  -> TMEM 128..255
//   softmax warps (thread = query slot): P = exp2(S scale log2e - LSE log2e) and
//     dS = P (dP - D) over the row's own keys, zeros elsewhere (each thread loads its query's
//     LSE and D = dO . O from global memory while the score MMAs run); P and dS (bf16) into shared memory
//     as [q][keys] panels, dS also into TMEM 448..511 as bf16 pairs
//   dV = P^T dO  (M=128 keys, N=64, K=128 q; A = P read MN-major, dO MN-major) -> 256..319
//   dK = dS^T Q  (same shapes, A = dS)                                          -> 320..383
//   dQ = dS K    (M=128 q, N=64, K=128 keys; A = dS from TMEM, K MN-major)      -> 384..447
//   epilogue warps (thread = token slot): dQ, dK (scaled) and dV in bf16 for slots < T.
// S / dP of item i + 1 are issued before the gradient MMAs of item i, so the softmax of the
// next item overlaps them; the epilogue warps drain the accumulators while the softmax
// warps work on the next item.
namespace fbw {
constexpr int kThreads = 320;                    // warps 0 (TMA), 1 (MMA), 2..5 softmax, 6..9 epilogue
constexpr int kStages = 2;                       // Q | K | V | dO per stage (64 KB)
constexpr int kPanel = 128 * 128;                // 16 KB: 128 query rows x 64 keys (bf16)
constexpr int kSmemBytes = kStages * 4 * ff::kTile + 4 * kPanel + 1024 + 256;
constexpr uint32_t kTmemCols = 512;
}  // namespace fbw

struct FeatBwdTcParams {
  int T, d_valid, H;
  int64_t n_rows, n_items;
  float scale, scale_log2;
  int q_pos[4], kv_pos[4], do_pos[4];
  const float* lse;   // [n_rows * H, T]
  const float* dvec;  // [n_rows * H, T]: dO . O per query
  __nv_bfloat16* dq;
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  int64_t g_s0, g_s2, g_row;  // dQ / dK / dV layout (shared)
  int* status;
};

__global__ void __launch_bounds__(fbw::kThreads, 1)
    attn_feat_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                            FeatBwdTcParams p) {
  using namespace fbw;
  constexpr int kTile = ff::kTile, kBox = ff::kBox;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sP = smem + kStages * 4 * kTile;  // 2 panels
  uint8_t* sDS = sP + 2 * kPanel;             // 2 panels
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDS + 2 * kPanel);
  uint64_t* kv_full = bars;             // [kStages]
  uint64_t* kv_empty = bars + kStages;  // [kStages]
  uint64_t* s_full = bars + 2 * kStages;
  uint64_t* s_free = s_full + 1;
  uint64_t* p_full = s_full + 2;
  uint64_t* pds_free = s_full + 3;
  uint64_t* acc_full = s_full + 4;
  uint64_t* acc_free = s_full + 5;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_full + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t n_items = p.n_items;
  if (p.status != nullptr && *reinterpret_cast<volatile int*>(p.status) != 0) return;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 4);
    mbar_init(p_full, 4);
    mbar_init(pds_free, 1);
    mbar_init(acc_full, 1);
    mbar_init(acc_free, 4);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tDP = tmem + 128, tDV = tmem + 256, tDK = tmem + 320, tDQ = tmem + 384,
                 tDS = tmem + 448;
  const int T = p.T;

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmDO);
      int it = 0;
      for (int64_t w = blockIdx.x; w < n_items; w += gridDim.x, ++it) {
        const int st = it % kStages;
        if (!mbar_wait(&kv_empty[st], ((it / kStages) & 1) ^ 1, p.status, kTimeoutProducer, abort_flag)) break;
        const int head = static_cast<int>(w % p.H);
        const int64_t row0 = (w / p.H) * 2;
        uint8_t* dst = smem + st * 4 * kTile;
        mbar_arrive_expect_tx(&kv_full[st], 4 * kTile);
        int c[5];
        for (int half = 0; half < 2; ++half) {
          feat_coords(p.q_pos, head, row0 + half, c);
          tma_load_5d(dst + half * kBox, &tmQ, &kv_full[st], c);
          feat_coords(p.kv_pos, head, row0 + half, c);
          tma_load_5d(dst + kTile + half * kBox, &tmK, &kv_full[st], c);
          tma_load_5d(dst + 2 * kTile + half * kBox, &tmV, &kv_full[st], c);
          feat_coords(p.do_pos, head, row0 + half, c);
          tma_load_5d(dst + 3 * kTile + half * kBox, &tmDO, &kv_full[st], c);
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t id_s = umma_idesc_bf16(128, 128, false, false);   // S, dP
      constexpr uint32_t id_kv = umma_idesc_bf16(128, ff::kD, true, true);  // dV, dK: A (P, dS) MN-major, B MN-major
      constexpr uint32_t id_q = umma_idesc_bf16(128, ff::kD, false, true);  // dQ: A = dS from TMEM, B MN-major
      const uint32_t aP = smem_u32(sP), aDS = smem_u32(sDS);
      bool ok = true;
      auto issue_grads = [&](int i) -> bool {
        const int st = i % kStages;
        if (!mbar_wait(p_full, i & 1, p.status, kTimeoutMma, abort_flag)) return false;
        if (i >= 1 && !mbar_wait(acc_free, (i - 1) & 1, p.status, kTimeoutMma, abort_flag)) return false;
        tc_fence_after();
        const uint32_t aQ = smem_u32(smem + st * 4 * kTile), aK = aQ + kTile, aDO = aQ + 3 * kTile;
#pragma unroll
        for (int k = 0; k < 128 / 16; ++k) {
          // A = P^T / dS^T [keys x q] read MN-major from the [q][keys] panels: 16 query rows
          // per step; B = dO / Q [q x d] MN-major
          umma_bf16_ss(tDV, umma_smem_desc(aP + k * 2048, kPanel, 1024, 2),
                       umma_smem_desc(aDO + k * 2048, 8192, 1024, 2), id_kv, k > 0 ? 1u : 0u);
          umma_bf16_ss(tDK, umma_smem_desc(aDS + k * 2048, kPanel, 1024, 2),
                       umma_smem_desc(aQ + k * 2048, 8192, 1024, 2), id_kv, k > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int k = 0; k < 128 / 16; ++k)
          umma_bf16_ts(tDQ, tDS + k * 8, umma_smem_desc(aK + k * 2048, 8192, 1024, 2), id_q, k > 0 ? 1u : 0u);
        umma_commit(acc_full);
        umma_commit(pds_free);
        umma_commit(&kv_empty[st]);
        return true;
      };
      int it = 0;
      for (int64_t w = blockIdx.x; ok && w < n_items; w += gridDim.x, ++it) {
        const int st = it % kStages;
        if (!(ok = mbar_wait(&kv_full[st], (it / kStages) & 1, p.status, kTimeoutMma, abort_flag))) break;
        // S / dP of this item overwrite the previous item's, which its softmax has read
        if (it >= 1 && !(ok = mbar_wait(s_free, (it - 1) & 1, p.status, kTimeoutMma, abort_flag))) break;
        tc_fence_after();
        const uint32_t aQ = smem_u32(smem + st * 4 * kTile), aK = aQ + kTile, aV = aQ + 2 * kTile,
                       aDO = aQ + 3 * kTile;
#pragma unroll
        for (int k = 0; k < ff::kD / 16; ++k) {
          umma_bf16_ss(tS, umma_desc_kmajor_sw128(aQ + k * 32), umma_desc_kmajor_sw128(aK + k * 32), id_s,
                       k > 0 ? 1u : 0u);
          umma_bf16_ss(tDP, umma_desc_kmajor_sw128(aDO + k * 32), umma_desc_kmajor_sw128(aV + k * 32), id_s,
                       k > 0 ? 1u : 0u);
        }
        umma_commit(s_full);
        if (it >= 1 && !(ok = issue_grads(it - 1))) break;
      }
      if (ok && it >= 1) issue_grads(it - 1);
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------ softmax: P, dS
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;  // MMA lane = query slot
    const int half = r >> 6, slot = r & 63;
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    constexpr float kLog2e = 1.4426950408889634f;
    bool ok = true;
    int it = 0;
    for (int64_t w = blockIdx.x; ok && w < n_items; w += gridDim.x, ++it) {
      // this query's -LSE log2e (-inf for a slot past T: P = 0) and D, loaded while the score
      // MMAs of the item run
      const int64_t row = (w / p.H) * 2 + half;
      const bool live = slot < T && row < p.n_rows;
      const int64_t vidx = (row * p.H + static_cast<int>(w % p.H)) * T + slot;
      const float nl = live ? -__ldg(p.lse + vidx) * kLog2e : -INFINITY;
      const float dd = live ? __ldg(p.dvec + vidx) : 0.f;
      if (!(ok = mbar_wait_warp(s_full, it & 1, p.status, kTimeoutEpilogue, abort_flag))) break;
      tc_fence_after();
      // P and dS in registers first (32 key columns at a time); the shared / tensor memory
      // they go to is still being read by the previous item's gradient MMAs
      uint32_t pk[32], dsk[32];
#pragma unroll
      for (int hk = 0; hk < 2; ++hk) {
        uint32_t sv[32], dpv[32];
        tmem_ld32(tS + lane_off + half * 64 + hk * 32, sv);
        tmem_ld32(tDP + lane_off + half * 64 + hk * 32, dpv);
        tmem_wait_ld();
#pragma unroll
        for (int j2 = 0; j2 < 16; ++j2) {
          float pe[2], de[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int jj = 2 * j2 + e;
            const float pv = hk * 32 + jj < T ? ex2_fast(fmaf(__uint_as_float(sv[jj]), p.scale_log2, nl)) : 0.f;
            pe[e] = pv;
            de[e] = pv * (__uint_as_float(dpv[jj]) - dd);
          }
          pk[hk * 16 + j2] = pack_bf16x2(pe[0], pe[1]);
          dsk[hk * 16 + j2] = pack_bf16x2(de[0], de[1]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);
      if (it >= 1 && !(ok = mbar_wait_warp(pds_free, (it - 1) & 1, p.status, kTimeoutEpilogue, abort_flag))) break;
      // this query row of the P / dS panels: its own row's keys in panel `half`, zeros in
      // the other panel (both 128B-swizzled K-major rows, conflict-free 16-byte stores)
      uint8_t* prow = sP + half * kPanel + r * 128;
      uint8_t* srow = sDS + half * kPanel + r * 128;
      uint8_t* prow0 = sP + (half ^ 1) * kPanel + r * 128;
      uint8_t* srow0 = sDS + (half ^ 1) * kPanel + r * 128;
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        const int sw = (ch ^ (r & 7)) << 4;
        *reinterpret_cast<uint4*>(prow + sw) = make_uint4(pk[4 * ch], pk[4 * ch + 1], pk[4 * ch + 2], pk[4 * ch + 3]);
        *reinterpret_cast<uint4*>(srow + sw) =
            make_uint4(dsk[4 * ch], dsk[4 * ch + 1], dsk[4 * ch + 2], dsk[4 * ch + 3]);
        *reinterpret_cast<uint4*>(prow0 + sw) = make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(srow0 + sw) = make_uint4(0u, 0u, 0u, 0u);
      }
      uint32_t zero[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) zero[j] = 0u;
      tmem_st32(tDS + lane_off + half * 32, dsk);
      tmem_st32(tDS + lane_off + (half ^ 1) * 32, zero);
      fence_proxy_async_smem();
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
  } else {
    // ------------------------------------------------------------ epilogue: dQ, dK, dV
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;  // token slot (query for dQ, key for dK / dV)
    const int half = r >> 6, slot = r & 63;
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    auto write_row = [&](__nv_bfloat16* base, int head, int64_t row, const uint32_t (&va)[32],
                         const uint32_t (&vb)[32], float mul) {
      __nv_bfloat16* out = base + row * p.g_s0 + static_cast<int64_t>(head) * p.g_s2 + slot * p.g_row;
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) {
        if (c8 * 8 >= p.d_valid) break;
        const uint32_t* src = c8 < 4 ? va + c8 * 8 : vb + (c8 - 4) * 8;
        *reinterpret_cast<uint4*>(out + c8 * 8) =
            make_uint4(pack_bf16x2(__uint_as_float(src[0]) * mul, __uint_as_float(src[1]) * mul),
                       pack_bf16x2(__uint_as_float(src[2]) * mul, __uint_as_float(src[3]) * mul),
                       pack_bf16x2(__uint_as_float(src[4]) * mul, __uint_as_float(src[5]) * mul),
                       pack_bf16x2(__uint_as_float(src[6]) * mul, __uint_as_float(src[7]) * mul));
      }
    };
    int it = 0;
    for (int64_t w = blockIdx.x; w < n_items; w += gridDim.x, ++it) {
      if (!mbar_wait_warp(acc_full, it & 1, p.status, kTimeoutEpilogue, abort_flag)) break;
      tc_fence_after();
      const int head = static_cast<int>(w % p.H);
      const int64_t row = (w / p.H) * 2 + half;
      const bool live = slot < T && row < p.n_rows;
      // one accumulator at a time (64 registers live); the last read frees the accumulators
      uint32_t va[32], vb[32];
      tmem_ld32(tDQ + lane_off, va);
      tmem_ld32(tDQ + 32 + lane_off, vb);
      tmem_wait_ld();
      if (live) write_row(p.dq, head, row, va, vb, p.scale);
      tmem_ld32(tDK + lane_off, va);
      tmem_ld32(tDK + 32 + lane_off, vb);
      tmem_wait_ld();
      if (live) write_row(p.dk, head, row, va, vb, p.scale);
      tmem_ld32(tDV + lane_off, va);
      tmem_ld32(tDV + 32 + lane_off, vb);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_free);  // the next item's gradient MMAs may start
      if (live) write_row(p.dv, head, row, va, vb, 1.f);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, fbw::kTmemCols);
  }
}

// ------------------------------------------------------------------ host
namespace {
// Feature layouts: (s0, s1, s2, row, d1, d2) = (T * width, *, head stride, width, 1, H).
void check_feat_layout(const std::vector<int64_t>& l, int64_t H, const char* what) {
  TORCH_CHECK(l.size() == 6 && l[4] == 1 && l[5] == H, what, ": feature layout (table row, head, token) expected");
}
int sm_count(int dev) {
  static int n_sm[64] = {0};
  if (n_sm[dev] == 0) C10_CUDA_CHECK(cudaDeviceGetAttribute(&n_sm[dev], cudaDevAttrMultiProcessorCount, dev));
  return n_sm[dev];
}
}  // namespace

torch::Tensor attn_dvec(const torch::Tensor& o, const torch::Tensor& dout, std::vector<int64_t> lo,
                        std::vector<int64_t> ldo, int64_t BH, int64_t Nq, int64_t d_valid);

bool attn_feat_tc_supported(int64_t T, int64_t d_valid) { return T >= 1 && T <= ff::kSlots && d_valid % 8 == 0 && d_valid <= ff::kD; }

void attn_feat_fwd_tc(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, torch::Tensor& o,
                      const c10::optional<torch::Tensor>& lse, std::vector<int64_t> lq, std::vector<int64_t> lk,
                      std::vector<int64_t> lv, std::vector<int64_t> lo, int64_t BH, int64_t T, int64_t d_valid,
                      double scale, const torch::Tensor& status) {
  for (const torch::Tensor* t : std::initializer_list<const torch::Tensor*>{&q, &k, &v, &o})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16, "attn_feat_fwd_tc: bf16 CUDA tensors");
  TORCH_CHECK(attn_feat_tc_supported(T, d_valid), "attn_feat_fwd_tc: rows of at most 64 tokens, head dim a multiple of 8 <= 64");
  const int64_t H = lq[5];
  check_feat_layout(lq, H, "attn_feat_fwd_tc q");
  check_feat_layout(lk, H, "attn_feat_fwd_tc k");
  check_feat_layout(lv, H, "attn_feat_fwd_tc v");
  check_feat_layout(lo, H, "attn_feat_fwd_tc o");
  for (int i = 0; i < 4; ++i) TORCH_CHECK(lo[i] % 8 == 0, "attn_feat_fwd_tc: output rows must be 16-byte aligned");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(o.data_ptr()) % 16 == 0, "attn_feat_fwd_tc: 16-byte aligned output");
  const at::cuda::CUDAGuard guard(q.device());
  if (BH == 0) return;
  TORCH_CHECK(BH % H == 0, "attn_feat_fwd_tc: BH must be table rows x heads");
  const int64_t n_rows = BH / H;
  TORCH_CHECK(n_rows < 2147483647LL, "attn_feat_fwd_tc: too many table rows");
  Map5 mq = make_map(q, lq, T, n_rows, static_cast<int>(d_valid), 2, ff::kD, ff::kSlots);
  Map5 mk = make_map(k, lk, T, n_rows, static_cast<int>(d_valid), 2, ff::kD, ff::kSlots);
  Map5 mv = make_map(v, lv, T, n_rows, static_cast<int>(d_valid), 2, ff::kD, ff::kSlots);
  TORCH_CHECK(std::equal(mk.pos, mk.pos + 4, mv.pos), "attn_feat_fwd_tc: K and V layouts must sort alike");
  FeatTcParams p{};
  p.T = static_cast<int>(T);
  p.d_valid = static_cast<int>(d_valid);
  p.H = static_cast<int>(H);
  p.n_rows = n_rows;
  p.n_items = ((n_rows + 1) / 2) * H;
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  std::copy(mq.pos, mq.pos + 4, p.q_pos);
  std::copy(mk.pos, mk.pos + 4, p.kv_pos);
  p.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.o_s0 = lo[0];
  p.o_s2 = lo[2];
  p.o_row = lo[3];
  if (lse.has_value() && lse->defined()) {
    TORCH_CHECK(lse->is_cuda() && lse->scalar_type() == at::kFloat && lse->numel() >= BH * T,
                "attn_feat_fwd_tc: fp32 lse [BH, T]");
    p.lse = lse->data_ptr<float>();
  }
  p.status = status.defined() && status.numel() > 0 ? status.data_ptr<int>() : nullptr;
  static bool configured[64] = {false};
  const int dev = q.get_device();
  if (!configured[dev]) {
    C10_CUDA_CHECK(
        cudaFuncSetAttribute(attn_feat_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ff::kSmemBytes));
    configured[dev] = true;
  }
  dim3 grid(static_cast<unsigned>(std::min<int64_t>(p.n_items, persistent_sms(sm_count(dev)))));
  attn_feat_fwd_tc_kernel<<<grid, ff::kThreads, ff::kSmemBytes, at::cuda::getCurrentCUDAStream()>>>(mq.map, mk.map,
                                                                                                   mv.map, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// dQ, dK, dV (bf16) share the layout lg; o / dout share lo.
void attn_feat_bwd_tc(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, const torch::Tensor& o,
                      const torch::Tensor& dout, const torch::Tensor& lse, torch::Tensor& dq, torch::Tensor& dk,
                      torch::Tensor& dv, std::vector<int64_t> lq, std::vector<int64_t> lkv, std::vector<int64_t> lo,
                      std::vector<int64_t> lg, int64_t BH, int64_t T, int64_t d_valid, double scale,
                      const torch::Tensor& status) {
  for (const torch::Tensor* t : std::initializer_list<const torch::Tensor*>{&q, &k, &v, &o, &dout, &dq, &dk, &dv})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16, "attn_feat_bwd_tc: bf16 CUDA tensors");
  TORCH_CHECK(lse.is_cuda() && lse.scalar_type() == at::kFloat && lse.numel() >= BH * T, "attn_feat_bwd_tc: fp32 lse [BH, T]");
  TORCH_CHECK(attn_feat_tc_supported(T, d_valid), "attn_feat_bwd_tc: rows of at most 64 tokens, head dim a multiple of 8 <= 64");
  const int64_t H = lq[5];
  check_feat_layout(lq, H, "attn_feat_bwd_tc q");
  check_feat_layout(lkv, H, "attn_feat_bwd_tc k/v");
  check_feat_layout(lo, H, "attn_feat_bwd_tc o/dout");
  check_feat_layout(lg, H, "attn_feat_bwd_tc dq/dk/dv");
  for (int i = 0; i < 4; ++i)
    TORCH_CHECK(lg[i] % 8 == 0 && lo[i] % 8 == 0, "attn_feat_bwd_tc: rows must be 16-byte aligned");
  for (const torch::Tensor* t : std::initializer_list<const torch::Tensor*>{&o, &dq, &dk, &dv})
    TORCH_CHECK(reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0, "attn_feat_bwd_tc: 16-byte aligned buffers");
  const at::cuda::CUDAGuard guard(q.device());
  if (BH == 0) return;
  TORCH_CHECK(BH % H == 0, "attn_feat_bwd_tc: BH must be table rows x heads");
  const int64_t n_rows = BH / H;
  TORCH_CHECK(n_rows < 2147483647LL, "attn_feat_bwd_tc: too many table rows");
  Map5 mq = make_map(q, lq, T, n_rows, static_cast<int>(d_valid), 2, ff::kD, ff::kSlots);
  Map5 mk = make_map(k, lkv, T, n_rows, static_cast<int>(d_valid), 2, ff::kD, ff::kSlots);
  Map5 mv = make_map(v, lkv, T, n_rows, static_cast<int>(d_valid), 2, ff::kD, ff::kSlots);
  Map5 mdo = make_map(dout, lo, T, n_rows, static_cast<int>(d_valid), 2, ff::kD, ff::kSlots);
  TORCH_CHECK(std::equal(mk.pos, mk.pos + 4, mv.pos), "attn_feat_bwd_tc: K and V layouts must sort alike");
  FeatBwdTcParams p{};
  p.T = static_cast<int>(T);
  p.d_valid = static_cast<int>(d_valid);
  p.H = static_cast<int>(H);
  p.n_rows = n_rows;
  p.n_items = ((n_rows + 1) / 2) * H;
  p.scale = static_cast<float>(scale);
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  std::copy(mq.pos, mq.pos + 4, p.q_pos);
  std::copy(mk.pos, mk.pos + 4, p.kv_pos);
  std::copy(mdo.pos, mdo.pos + 4, p.do_pos);
  p.lse = lse.data_ptr<float>();
  // D = dO . O per query (one memory-bound pass; the kernel stages it per item with the LSE)
  const torch::Tensor dvec = attn_dvec(o, dout, lo, lo, BH, T, d_valid);
  p.dvec = dvec.data_ptr<float>();
  p.dq = reinterpret_cast<__nv_bfloat16*>(dq.data_ptr());
  p.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  p.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  p.g_s0 = lg[0];
  p.g_s2 = lg[2];
  p.g_row = lg[3];
  p.status = status.defined() && status.numel() > 0 ? status.data_ptr<int>() : nullptr;
  static bool configured[64] = {false};
  const int dev = q.get_device();
  if (!configured[dev]) {
    C10_CUDA_CHECK(
        cudaFuncSetAttribute(attn_feat_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, fbw::kSmemBytes));
    configured[dev] = true;
  }
  dim3 grid(static_cast<unsigned>(std::min<int64_t>(p.n_items, persistent_sms(sm_count(dev)))));
  attn_feat_bwd_tc_kernel<<<grid, fbw::kThreads, fbw::kSmemBytes, at::cuda::getCurrentCUDAStream()>>>(
      mq.map, mk.map, mv.map, mdo.map, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace nori
