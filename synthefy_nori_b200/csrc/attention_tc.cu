// Flash attention forward on the 5th-generation tensor cores (tcgen05 + TMEM + TMA),
// used for the long sequence (ICL) attention of the Nori encoder: context
// self-attention and query->context cross-attention per (table, column, head)
// (reference model/layer.py:1407-1441, 685-745).
//
// Persistent: one CTA per SM loops over work items (one item = 128 query rows of one
// head); TMEM, barriers and the K / V pipeline carry over from item to item, so the next
// item's Q and K / V loads overlap the current item's last tiles.  Warp roles (384 threads):
//   warp 0      TMA producer: the Q tile once, then 128-key K and V tiles into two
//               3-stage rings (K(j) is released when S_j completes, V(j) when O_j
//               completes; 5-D tensor maps read the strided token-major layouts
//               directly; head-dim padding and tails are zero-filled by TMA);
//   warp 1      TMEM owner + MMA issuer: S_j = Q K_j^T (M=128, N=128, K=64) into the
//               score buffer of group j % 2, then O_g += P_j V_j (M=128, N=64, K=128,
//               V read MN-major) into that group's TMEM accumulator; order S_0, S_1,
//               PV_0, S_2, PV_1, S_3, ... so a score tile is always in flight;
//   warps 4..7 / 8..11  two softmax groups, one per key-tile parity, each with its own
//               running max / sum: thread = query row (its TMEM lane), all 128 columns;
//               P_j (bf16 pairs) is stored back over the first 64 columns of its own score
//               buffer in TMEM, and the P . V MMA takes its A operand from there (no
//               shared-memory round trip for P: the tensor cores read only V from shared
//               memory for that product).  The max is lazy (O_g is rescaled in TMEM only when a row's
//               max grows by more than 2^8), and the groups merge their (max, sum,
//               O_g) once per item.  The two groups work on different tiles at the same
//               time, so one group's waits overlap the other's arithmetic.
// Every mbarrier wait is bounded (see sm100.cuh); on timeout the CTA records an error
// in the status word and returns after freeing its TMEM.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <algorithm>
#include <array>

#include "sm100.cuh"
#include "tma_host.h"

namespace nori {

namespace fa {
constexpr int kM = 128;      // query rows per CTA
constexpr int kN = 128;      // keys per tile
constexpr int kD = 64;       // padded head dim
constexpr int kThreads = 384;  // warps 0 (TMA), 1 (MMA), 4..11 (softmax)

constexpr int kSoftmaxWarps = 8;  // softmax-side barriers take one arrive per warp
// register split of the forward kernel (launch: 384 threads x 168 = 64512), made inside each
// role's branch: warps 0..3 (TMA, MMA, two idle) give up to kRegsLow, the eight softmax
// warps take kRegsSoftmax
constexpr uint32_t kRegsLow = 48, kRegsSoftmax = 224;
static_assert(4 * 32 * kRegsLow + 8 * 32 * kRegsSoftmax <= kThreads * 168, "register split over the launch total");
constexpr int kTileBytes = kM * kD * 2;  // 16 KB (Q, K or V tile)
constexpr int kStages = 3;  // K and V rings (separate: K(j) frees after S_j, V(j) after O_j)
// smem: Q[2] | K[3] | V[3] | barriers
constexpr int kSmemBytes = kTileBytes * (2 + 2 * kStages) + 1024 + 256;
// S[2] (2 x 128; P_j overwrites the first 64 columns of its S buffer) + O[item parity][group] (4 x 64)
constexpr uint32_t kTmemCols = 512;
}  // namespace fa

struct AttnTcParams {
  int Nq, Nk, d_valid;
  int n_tiles_q;
  int64_t n_items;  // BH * n_tiles_q work items (head, query tile), visited with stride gridDim.x
  float scale_log2;
  // coordinate positions (inside the 5-D maps) of row / i2 / i1 / i0 for Q and for K/V
  int q_pos[4], kv_pos[4];
  int d1, d2;  // bh decomposition
  __nv_bfloat16* o;
  int64_t o_s0, o_s1, o_s2, o_row;
  float* lse;
  int* status;
};

// 2^x for x <= 0 without the XU pipe (the MUFU, float->int conversions and rounding all
// issue there, and the softmax already keeps it busy with ex2 and bf16 packing):
//   t = x + 1.5 * 2^23 rounds x to the nearest integer n, which then sits in the low
//   mantissa bits of t (FADD); f = x - n in [-0.5, 0.5];
//   2^f ~ c0 + c1 f + c2 f^2 + c3 f^3 (minimax in relative error on [-0.5, 0.5], fitted for
//   this kernel: max relative error 7.5e-5, well under bf16's 2^-9);
//   2^n enters as (bits of t) << 23 added to the exponent field (integer ALU).
// x is clamped at -125 so the scaled result stays a normal float.
__device__ __forceinline__ float exp2_poly(float x) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  x = fmaxf(x, -125.0f);
  const float t = x + kRound;
  const float f = x - (t - kRound);
  float pl = fmaf(f, 0.0551716648042202f, 0.2426111251115799f);
  pl = fmaf(pl, f, 0.6932609677314758f);
  pl = fmaf(pl, f, 0.9999280571937561f);
  return __uint_as_float(__float_as_uint(pl) + (__float_as_uint(t) << 23));
}

// 2^x on the MUFU (one instruction; flushes subnormal results to zero, which the bf16 P
// cannot represent anyway).
__device__ __forceinline__ float exp2_mufu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pairs (sm_100 f32x2 instructions: two lanes of FMA-pipe work per issue).
__device__ __forceinline__ uint64_t f2pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// exp2_poly on a packed pair: the rounding, reduction and polynomial run as f32x2.
__device__ __forceinline__ void exp2_poly2(uint64_t x2, float& e0, float& e1) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  float x0, x1;
  f2unpack(x2, x0, x1);
  x2 = f2pack(fmaxf(x0, -125.0f), fmaxf(x1, -125.0f));
  const uint64_t r2 = f2pack(kRound, kRound);
  const uint64_t t2 = f2add(x2, r2);
  const uint64_t f2 = f2sub(x2, f2sub(t2, r2));
  uint64_t pl = f2fma(f2, f2pack(0.0551716648042202f, 0.0551716648042202f),
                      f2pack(0.2426111251115799f, 0.2426111251115799f));
  pl = f2fma(pl, f2, f2pack(0.6932609677314758f, 0.6932609677314758f));
  pl = f2fma(pl, f2, f2pack(0.9999280571937561f, 0.9999280571937561f));
  float p0, p1, t0, t1;
  f2unpack(pl, p0, p1);
  f2unpack(t2, t0, t1);
  e0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
  e1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
}

__device__ __forceinline__ void coords_for(const int (&pos)[4], int row, int i2, int i1, int i0, int (&c)[5]) {
  c[0] = 0;
  c[pos[0]] = row;
  c[pos[1]] = i2;
  c[pos[2]] = i1;
  c[pos[3]] = i0;
}

// Row maximum of 64 score columns (two 32-column TMEM loads), `valid` of them real.
__device__ __forceinline__ float rowmax64(const uint32_t (&va)[32], const uint32_t (&vb)[32], int valid) {
  if (valid >= 64) {
    float m8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      m8[i] = fmax3(__uint_as_float(va[i]), __uint_as_float(va[i + 8]), __uint_as_float(va[i + 16]));
#pragma unroll
    for (int i = 0; i < 8; ++i)
      m8[i] = fmax3(m8[i], __uint_as_float(va[i + 24]), __uint_as_float(vb[i]));
#pragma unroll
    for (int i = 0; i < 8; ++i)
      m8[i] = fmax3(m8[i], __uint_as_float(vb[i + 8]), __uint_as_float(vb[i + 16]));
#pragma unroll
    for (int i = 0; i < 8; ++i) m8[i] = fmaxf(m8[i], __uint_as_float(vb[i + 24]));
    return fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
  }
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    if (i < valid) m = fmaxf(m, __uint_as_float(va[i]));
    if (32 + i < valid) m = fmaxf(m, __uint_as_float(vb[i]));
  }
  return m;
}

// P = 2^(s scale_log2 + nm) for 32 score columns -> 16 packed bf16 pairs; returns the row
// sum of the (fp32) values. Columns at or past `valid` give 0.
__device__ __forceinline__ float softmax_chunk32(const uint32_t (&v)[32], int valid, float scale_log2, float nm,
                                                 uint32_t (&pk)[16]) {
  if (valid >= 32) {
    const uint64_t sc2 = f2pack(scale_log2, scale_log2), nm2 = f2pack(nm, nm);
    uint64_t rsa = 0, rsb = 0;  // packed partial row sums (+0.0f, +0.0f)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      // columns 4i, 4i+1 on the MUFU, 4i+2, 4i+3 on the FMA pipe (polynomial 2^x)
      const uint64_t xa = f2fma(f2pack(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1])), sc2, nm2);
      const uint64_t xb = f2fma(f2pack(__uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3])), sc2, nm2);
      float xa0, xa1, e2, e3;
      f2unpack(xa, xa0, xa1);
      const float e0 = exp2_mufu(xa0), e1 = exp2_mufu(xa1);
      exp2_poly2(xb, e2, e3);
      pk[2 * i] = pack_bf16x2(e0, e1);
      pk[2 * i + 1] = pack_bf16x2(e2, e3);
      rsa = f2add(rsa, f2pack(e0, e1));
      rsb = f2add(rsb, f2pack(e2, e3));
    }
    float r0, r1;
    f2unpack(f2add(rsa, rsb), r0, r1);
    return r0 + r1;
  }
  float rs = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float e0 = 2 * i < valid ? exp2_mufu(fmaf(__uint_as_float(v[2 * i]), scale_log2, nm)) : 0.f;
    const float e1 = 2 * i + 1 < valid ? exp2_mufu(fmaf(__uint_as_float(v[2 * i + 1]), scale_log2, nm)) : 0.f;
    pk[i] = pack_bf16x2(e0, e1);
    rs += e0 + e1;
  }
  return rs;
}

__global__ void __launch_bounds__(fa::kThreads, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, AttnTcParams p) {
  using namespace fa;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                             // 2 buffers (consecutive work items)
  uint8_t* sK = sQ + 2 * kTileBytes;              // kStages
  uint8_t* sV = sK + kStages * kTileBytes;        // kStages
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kStages * kTileBytes);
  uint64_t* q_full = bars;        // [2]
  uint64_t* q_empty = bars + 2;   // [2]
  uint64_t* s_full = bars + 4;    // [group]
  uint64_t* p_full = bars + 6;    // [group]
  uint64_t* o_full = bars + 8;    // [group]
  uint64_t* o_free = bars + 10;   // [item parity] that item's accumulators read by its epilogue
  uint64_t* sbar = bars + 12;     // [item parity] (max, sum) exchange at the end of an item
  uint64_t* k_full = bars + 14;   // [kStages]
  uint64_t* k_empty = bars + 17;  // [kStages]
  uint64_t* v_full = bars + 20;   // [kStages]
  uint64_t* v_empty = bars + 23;  // [kStages]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 26);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  __shared__ float red_m[2][2][kM];  // [item parity][group][row]
  __shared__ float red_l[2][2][kM];

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_tiles = (p.Nk + kN - 1) / kN;
  const int64_t n_items = p.n_items;
  // a CTA that starts after another one timed out returns at once
  if (p.status != nullptr && *reinterpret_cast<volatile int*>(p.status) != 0) return;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], kSoftmaxWarps / 2);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], kSoftmaxWarps);
      mbar_init(&sbar[i], kSoftmaxWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem;            // S buffers (one per group) at columns 0, 128
  // O accumulators: two sets (item parity) of one per group, at columns 256 + 128 set + 64 group,
  // so the next item's P . V products overlap this item's epilogue
  const uint32_t tO = tmem + 2 * kN;

  // work item w -> (head bh, query tile); items are visited with stride gridDim.x
  auto item_coords = [&](int64_t w, int& q0, int& i2, int& i1, int& i0, int64_t& bh) {
    bh = w / p.n_tiles_q;
    q0 = static_cast<int>(w % p.n_tiles_q) * kM;
    i2 = static_cast<int>(bh % p.d2);
    i1 = static_cast<int>((bh / p.d2) % p.d1);
    i0 = static_cast<int>(bh / (static_cast<int64_t>(p.d1) * p.d2));
  };

  if (warp == 0) {
    setmaxnreg_dec<kRegsLow>();
    if (elect_one()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      int c[5];
      int64_t gk = 0, gv = 0;  // global K / V tile counters (ring positions)
      int it = 0;
      bool pok = true;
      for (int64_t w = blockIdx.x; pok && w < n_items; w += gridDim.x, ++it) {
        int q0, i2, i1, i0;
        int64_t bh;
        item_coords(w, q0, i2, i1, i0, bh);
        const int qb = it & 1;
        if (!mbar_wait(&q_empty[qb], ((it >> 1) & 1) ^ 1, p.status, kTimeoutProducer, abort_flag)) break;
        coords_for(p.q_pos, q0, i2, i1, i0, c);
        mbar_arrive_expect_tx(&q_full[qb], kTileBytes);
        tma_load_5d(sQ + qb * kTileBytes, &tmQ, &q_full[qb], c);
        // K(j) can be reloaded once S_j is done, V(j) once O_j is done; K runs one tile
        // ahead of V so a slow V slot never holds back the next score tile
        auto load_k = [&](int j) -> bool {
          const int st = static_cast<int>(gk % kStages);
          if (!mbar_wait(&k_empty[st], ((gk / kStages) & 1) ^ 1, p.status, kTimeoutProducer, abort_flag)) return false;
          coords_for(p.kv_pos, j * kN, i2, i1, i0, c);
          mbar_arrive_expect_tx(&k_full[st], kTileBytes);
          tma_load_5d(sK + st * kTileBytes, &tmK, &k_full[st], c);
          ++gk;
          return true;
        };
        pok = load_k(0);
        for (int j = 0; pok && j < n_tiles; ++j) {
          if (j + 1 < n_tiles && !(pok = load_k(j + 1))) break;
          const int st = static_cast<int>(gv % kStages);
          if (!(pok = mbar_wait(&v_empty[st], ((gv / kStages) & 1) ^ 1, p.status, kTimeoutProducer, abort_flag)))
            break;
          coords_for(p.kv_pos, j * kN, i2, i1, i0, c);
          mbar_arrive_expect_tx(&v_full[st], kTileBytes);
          tma_load_5d(sV + st * kTileBytes, &tmV, &v_full[st], c);
          ++gv;
        }
      }
    }
  } else if (warp == 1) {
    setmaxnreg_dec<kRegsLow>();
    if (elect_one()) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(kM, kN, false, false);
      constexpr uint32_t idesc_o = umma_idesc_bf16(kM, kD, false, true);
      int64_t gk = 0, gv = 0;     // K / V ring positions
      int64_t cnt[2] = {0, 0};    // tiles per group so far (s_full / p_full / o_full completions)
      int it = 0;
      bool ok = true;
      for (int64_t w = blockIdx.x; ok && w < n_items; w += gridDim.x, ++it) {
        const int qb = it & 1;
        if (!(ok = mbar_wait(&q_full[qb], (it >> 1) & 1, p.status, kTimeoutMma, abort_flag))) break;
        const uint32_t aQ = smem_u32(sQ + qb * kTileBytes);
        // S of the group's next key tile into that group's score buffer
        auto issue_s = [&](int grp) -> bool {
          const int st = static_cast<int>(gk % kStages);
          if (!mbar_wait(&k_full[st], (gk / kStages) & 1, p.status, kTimeoutMma, abort_flag)) return false;
          tc_fence_after();
          const uint32_t bK = smem_u32(sK + st * kTileBytes);
#pragma unroll
          for (int k = 0; k < kD / 16; ++k)
            umma_bf16_ss(tS + grp * kN, umma_desc_kmajor_sw128(aQ + k * 32), umma_desc_kmajor_sw128(bK + k * 32),
                         idesc_s, k > 0 ? 1u : 0u);
          umma_commit(&s_full[grp]);
          umma_commit(&k_empty[st]);
          ++gk;
          return true;
        };
        ok = issue_s(0);
        if (ok && n_tiles > 1) ok = issue_s(1);
        if (ok && n_tiles <= 2) umma_commit(&q_empty[qb]);  // every score MMA of the item read Q
        for (int j = 0; ok && j < n_tiles; ++j) {
          const int grp = j & 1;
          const bool first = j < 2;  // the group's first tile of this item starts its accumulator
          if (!(ok = mbar_wait(&p_full[grp], cnt[grp] & 1, p.status, kTimeoutMma, abort_flag))) break;
          if (first && it >= 2 &&
              !(ok = mbar_wait(&o_free[qb], ((it >> 1) - 1) & 1, p.status, kTimeoutMma, abort_flag)))
            break;
          const int st = static_cast<int>(gv % kStages);
          if (!(ok = mbar_wait(&v_full[st], (gv / kStages) & 1, p.status, kTimeoutMma, abort_flag))) break;
          tc_fence_after();
          const uint32_t bV = smem_u32(sV + st * kTileBytes);
          // A = P_j from TMEM (8 columns of bf16 pairs per 16 keys); this MMA is issued before
          // the group's next score MMA, which overwrites the same columns, and tcgen05.mma of
          // one thread execute in issue order
#pragma unroll
          for (int k = 0; k < kN / 16; ++k) {
            const uint64_t db = umma_smem_desc(bV + k * 2048, 8192, 1024, 2);
            umma_bf16_ts(tO + (qb * 2 + grp) * kD, tS + grp * kN + k * 8, db, idesc_o, (k > 0 || !first) ? 1u : 0u);
          }
          umma_commit(&o_full[grp]);
          umma_commit(&v_empty[st]);
          ++gv;
          ++cnt[grp];
          if (j + 2 < n_tiles) {
            ok = issue_s(grp);
            if (ok && j + 2 == n_tiles - 1) umma_commit(&q_empty[qb]);
          }
        }
      }
    }
  } else if (warp < 4) {
    setmaxnreg_dec<kRegsLow>();  // idle warps 2, 3 take part in their warpgroup's split
  } else {
    setmaxnreg_inc<kRegsSoftmax>();
    // ------------------------------------------------------------ softmax
    // Group g (warps 4..7 -> 0, 8..11 -> 1) takes the key tiles j = g, g + 2, ... of each
    // item with its own running max / sum and its own TMEM accumulator O_g; thread = query
    // row (its TMEM lane), all 128 score columns. The max is lazy: O_g and the sum are
    // rescaled only when a row's max grows by more than 2^8, so P values stay <= 256
    // (exact enough in bf16) and most tiles skip the rescale. At the end of the item the
    // two groups exchange (max, sum) and each writes half of the output columns from
    // both accumulators.
    constexpr float kRescaleLog2 = 8.0f;
    const int grp = (warp - 4) >> 2;
    const int q = warp & 3;
    const int r = q * 32 + lane;  // row in tile == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t tSg = tS + grp * kN + lane_off;
    bool ok = true;
    int64_t cnt = 0;  // this group's tiles so far (barrier completions)
    int it = 0;
    for (int64_t w = blockIdx.x; ok && w < n_items; w += gridDim.x, ++it) {
      int q0, i2, i1, i0;
      int64_t bh;
      item_coords(w, q0, i2, i1, i0, bh);
      const uint32_t tOi = tO + (it & 1) * 2 * kD;  // this item's accumulator set
      const uint32_t tOg = tOi + grp * kD + lane_off;
      float m_used = -INFINITY, l = 0.f;
      for (int j = grp; ok && j < n_tiles; j += 2, ++cnt) {
        if (!mbar_wait_warp(&s_full[grp], cnt & 1, p.status, kTimeoutEpilogue, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int valid = min(kN, p.Nk - j * kN);
        // the whole 128-column score row in registers (one TMEM round trip)
        uint32_t va[32], vb[32], vc[32], vd[32];
        tmem_ld32(tSg, va);
        tmem_ld32(tSg + 32, vb);
        tmem_ld32(tSg + 64, vc);
        tmem_ld32(tSg + 96, vd);
        tmem_wait_ld();
        float mx = rowmax64(va, vb, valid);
        if (valid > 64) mx = fmaxf(mx, rowmax64(vc, vd, valid - 64));
        const float m_cand = mx * p.scale_log2;
        // the group's previous P . V (same accumulator) must be complete before O is
        // rescaled (it is: s_full of this tile was committed after it; the wait also orders
        // the accumulator reads below)
        if (cnt > 0 && !mbar_wait_warp(&o_full[grp], (cnt - 1) & 1, p.status, kTimeoutEpilogue, abort_flag)) {
          ok = false;
          break;
        }
        float a = 1.f;
        bool need = false;
        if (j == grp) {
          m_used = m_cand;  // first tile: the accumulator starts fresh
        } else if (m_cand > m_used + kRescaleLog2) {
          a = exp2f(m_used - m_cand);
          m_used = m_cand;
          need = true;
        }
        // P (bf16 pairs) over the first 64 columns of this group's score buffer: keys
        // 32c .. 32c + 31 go to columns 16c .. 16c + 15 (the whole row is in registers already)
        const float nm = -m_used;
        float rsum = 0.f;
        {
          uint32_t pk[16];
          rsum += softmax_chunk32(va, valid, p.scale_log2, nm, pk);
          tmem_st16(tSg, pk);
          rsum += softmax_chunk32(vb, valid - 32, p.scale_log2, nm, pk);
          tmem_st16(tSg + 16, pk);
          rsum += softmax_chunk32(vc, valid - 64, p.scale_log2, nm, pk);
          tmem_st16(tSg + 32, pk);
          rsum += softmax_chunk32(vd, valid - 96, p.scale_log2, nm, pk);
          tmem_st16(tSg + 48, pk);
        }
        // O_g rescale after P left the registers (warp-collective TMEM read-modify-write;
        // lanes that keep their max scale by 1)
        if (__any_sync(0xffffffffu, need)) {
          tc_fence_after();
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t o[32];
            tmem_ld32(tOg + h * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * a);
            tmem_st32(tOg + h * 32, o);
          }
          tmem_wait_st();
        }
        l = l * a;
        l += rsum;
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[grp]);
      }
      // epilogue: this group's last P . V done, exchange (max, sum), combine the accumulators
      const bool has1 = n_tiles > 1;
      if (ok && (grp == 0 || has1))
        ok = mbar_wait_warp(&o_full[grp], (cnt - 1) & 1, p.status, kTimeoutEpilogue, abort_flag);
      red_m[it & 1][grp][r] = m_used;
      red_l[it & 1][grp][r] = l;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sbar[it & 1]);
      if (ok) ok = mbar_wait_warp(&sbar[it & 1], (it >> 1) & 1, p.status, kTimeoutEpilogue, abort_flag);
      if (ok) {
        tc_fence_after();
        const float m0 = red_m[it & 1][0][r], l0 = red_l[it & 1][0][r];
        const float m1 = has1 ? red_m[it & 1][1][r] : -INFINITY, l1 = has1 ? red_l[it & 1][1][r] : 0.f;
        const float m = fmaxf(m0, m1);
        const float f0 = exp2f(m0 - m), f1 = has1 ? exp2f(m1 - m) : 0.f;
        const float lt = l0 * f0 + l1 * f1;
        uint32_t a0[32], a1[32];
        tmem_ld32(tOi + lane_off + grp * 32, a0);
        if (has1) tmem_ld32(tOi + kD + lane_off + grp * 32, a1);
        tmem_wait_ld();
        const int row = q0 + r;
        if (row < p.Nq) {
          const float inv = lt > 0.f ? 1.f / lt : 0.f;
          const float g0 = f0 * inv, g1 = f1 * inv;
          float o[32];
#pragma unroll
          for (int i = 0; i < 32; ++i)
            o[i] = __uint_as_float(a0[i]) * g0 + (has1 ? __uint_as_float(a1[i]) * g1 : 0.f);
          __nv_bfloat16* out = p.o + static_cast<int64_t>(i0) * p.o_s0 + static_cast<int64_t>(i1) * p.o_s1 +
                               static_cast<int64_t>(i2) * p.o_s2 + static_cast<int64_t>(row) * p.o_row + grp * 32;
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            if (grp * 32 + c8 * 8 < p.d_valid) {
              *reinterpret_cast<uint4*>(out + c8 * 8) =
                  make_uint4(pack_bf16x2(o[c8 * 8], o[c8 * 8 + 1]), pack_bf16x2(o[c8 * 8 + 2], o[c8 * 8 + 3]),
                             pack_bf16x2(o[c8 * 8 + 4], o[c8 * 8 + 5]), pack_bf16x2(o[c8 * 8 + 6], o[c8 * 8 + 7]));
            }
          }
          if (p.lse != nullptr && grp == 0) {
            constexpr float kLn2 = 0.6931471805599453f;
            p.lse[bh * p.Nq + row] = lt > 0.f ? (m + log2f(lt)) * kLn2 : -INFINITY;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&o_free[it & 1]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------ backward
// Persistent: one CTA per SM loops over work items (one item = 128 keys of one head;
// dK / dV in TMEM are handed back through acc_free).  Per item, loop over 128-row query
// blocks:
//   S^T  = K Q^T     (M=128 keys, N=128 q, K=64)   -> TMEM
//   dP^T = V dO^T    (M=128 keys, N=128 q, K=64)   -> TMEM
//   softmax warps (thread = key row, two warps per lane quarter split the q columns):
//     P^T = exp2(S^T scale log2e - LSE log2e) -> bf16 pairs into 64 TMEM columns,
//     dS^T = P^T (dP^T - Dvec) -> bf16, smem
//   dV += P^T dO     (M=128 keys, N=64, K=128 q; A = P^T from TMEM, dO read MN-major)
//   dK += dS^T Q     (M=128 keys, N=64, K=128 q; Q read MN-major)
//   dQ  = dS K       (M=128 q, N=64, K=128 keys; dS^T read MN-major as A, K MN-major)
//   the softmax warps drain dQ (thread = query row) into a 4 KB shared-memory slot per
//   warp and add it to the caller's zeroed fp32 accumulator with one TMA tensor
//   reduce-add per warp (the additions happen in L2), and finally write dK (scaled) and dV.
namespace fb {
constexpr int kM = 128, kD = 64;
constexpr int kThreads = 384;  // warps 0 (TMA), 1 (MMA), 4..11 (softmax / drain)
constexpr int kWarpsSm = 8;
constexpr int kTile = kM * kD * 2;      // 16 KB
constexpr int kPanel = kM * 128;        // 16 KB: 128 rows x 64 bf16
// smem: K | V | Q[2] | dO[2] | dS^T (2 panels) | dQ staging (8 x 4 KB) | barriers
constexpr int kDQStage = 32 * 128;      // 4 KB per drain warp: 32 query rows x 32 fp32 (128B-swizzled)
constexpr int kSmemBytes = kTile * 6 + 2 * kPanel + kWarpsSm * kDQStage + 1024 + 256;
// S 0..127, dP 128..255, dV 256..319, dK 320..383, dQ 384..447, P^T (bf16 pairs) 448..511
constexpr uint32_t kTmemCols = 512;
}  // namespace fb

struct AttnBwdTcParams {
  int Nq, Nk, d_valid;
  int n_tiles_k;
  int64_t n_items;  // BH * n_tiles_k work items (head, key tile), visited with stride gridDim.x
  float scale, scale_log2;
  int q_pos[4], kv_pos[4], dq_pos[4];
  int d1, d2;
  const float* lse;   // [BH, Nq]
  const float* dvec;  // [BH, Nq]
  float* dq;          // fp32 accumulator: (i0, i1, i2, row) strides dq_s0.. dq_row
  int64_t dq_s0, dq_s1, dq_s2, dq_row;
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  int64_t kv_s0, kv_s1, kv_s2, kv_row;  // dK / dV layout
  int* status;
};


__global__ void __launch_bounds__(fb::kThreads, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                       const __grid_constant__ CUtensorMap tmDQ, AttnBwdTcParams p) {
  using namespace fb;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + kTile;
  uint8_t* sQ = sV + kTile;        // 2 stages
  uint8_t* sDO = sQ + 2 * kTile;   // 2 stages
  uint8_t* sDS = sDO + 2 * kTile;  // 2 panels
  uint8_t* sDQ = sDS + 2 * kPanel; // dQ staging, one 4 KB slot per drain warp
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDQ + kWarpsSm * kDQStage);
  uint64_t* kv_full = bars;        // [1] (index 1 unused)
  uint64_t* kv_empty = bars + 2;   // [1]
  uint64_t* qd_full = bars + 4;    // [2]
  uint64_t* qd_empty = bars + 6;   // [2]
  uint64_t* s_full = bars + 8;
  uint64_t* s_free = bars + 9;
  uint64_t* p_full = bars + 10;
  uint64_t* pds_free = bars + 11;
  uint64_t* dq_full = bars + 12;
  uint64_t* dq_free = bars + 13;
  uint64_t* acc_full = bars + 14;
  uint64_t* acc_free = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // per-stage query vectors: LSE (log2 units) and Dvec of the block's 128 queries
  __shared__ __align__(16) float s_lse[2][kM];
  __shared__ __align__(16) float s_dv[2][kM];

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_qt = (p.Nq + kM - 1) / kM;
  const int64_t n_items = p.n_items;
  if (p.status != nullptr && *reinterpret_cast<volatile int*>(p.status) != 0) return;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&qd_full[i], 2);  // TMA (expect_tx) + the producer warp's vector loads
      mbar_init(&qd_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, kWarpsSm);
    mbar_init(p_full, kWarpsSm);
    mbar_init(pds_free, 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, kWarpsSm);
    mbar_init(acc_full, 1);
    mbar_init(acc_free, kWarpsSm);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tDP = tmem + 128, tDV = tmem + 256, tDK = tmem + 320, tDQ = tmem + 384;
  const uint32_t tPT = tmem + 448;  // P^T: key row = lane, queries 2c, 2c + 1 in column c

  // work item w -> (head bh, key tile); items are visited with stride gridDim.x
  auto item_coords = [&](int64_t w, int& k0, int& i2, int& i1, int& i0, int64_t& bh) {
    bh = w / p.n_tiles_k;
    k0 = static_cast<int>(w % p.n_tiles_k) * kM;
    i2 = static_cast<int>(bh % p.d2);
    i1 = static_cast<int>((bh / p.d2) % p.d1);
    i0 = static_cast<int>(bh / (static_cast<int64_t>(p.d1) * p.d2));
  };

  if (warp == 0) {
    // whole warp: lane 0 issues the TMA loads, all lanes stage LSE / Dvec of the block
    constexpr float kLog2e = 1.4426950408889634f;
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmDO);
    }
    int64_t gq = 0;  // global query-block counter (Q / dO stages)
    int it = 0;
    bool pok = true;
    for (int64_t w = blockIdx.x; pok && w < n_items; w += gridDim.x, ++it) {
      int k0, i2, i1, i0;
      int64_t bh;
      item_coords(w, k0, i2, i1, i0, bh);
      const int kb = 0;  // one K / V buffer: the next item's load waits for this item's last MMA
      if (!(pok = mbar_wait_warp(&kv_empty[kb], (it & 1) ^ 1, p.status, kTimeoutProducer, abort_flag))) break;
      if (lane == 0) {
        int c[5];
        coords_for(p.kv_pos, k0, i2, i1, i0, c);
        mbar_arrive_expect_tx(&kv_full[kb], 2 * kTile);
        tma_load_5d(sK + kb * kTile, &tmK, &kv_full[kb], c);
        tma_load_5d(sV + kb * kTile, &tmV, &kv_full[kb], c);
      }
      const float* lse_g = p.lse + bh * p.Nq;
      const float* dv_g = p.dvec + bh * p.Nq;
      for (int j = 0; j < n_qt; ++j, ++gq) {
        const int s = static_cast<int>(gq & 1);
        if (!(pok = mbar_wait_warp(&qd_empty[s], ((gq >> 1) & 1) ^ 1, p.status, kTimeoutProducer, abort_flag))) break;
        if (lane == 0) {
          int c[5];
          coords_for(p.q_pos, j * kM, i2, i1, i0, c);
          mbar_arrive_expect_tx(&qd_full[s], 2 * kTile);
          tma_load_5d(sQ + s * kTile, &tmQ, &qd_full[s], c);
          tma_load_5d(sDO + s * kTile, &tmDO, &qd_full[s], c);
        }
        for (int i = lane; i < kM; i += 32) {
          const int qi = j * kM + i;
          s_lse[s][i] = qi < p.Nq ? -lse_g[qi] * kLog2e : -INFINITY;  // negated: added in the exponent
          s_dv[s][i] = qi < p.Nq ? dv_g[qi] : 0.f;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&qd_full[s]);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t id_s = umma_idesc_bf16(kM, kM, false, false);    // S^T, dP^T
      constexpr uint32_t id_kv = umma_idesc_bf16(kM, kD, false, true);    // dV, dK: A K-major, B MN-major
      constexpr uint32_t id_q = umma_idesc_bf16(kM, kD, true, true);      // dQ: A (dS) MN-major, B (K) MN-major
      const uint32_t aDS = smem_u32(sDS);
      int64_t gq = 0;  // global query-block counter: Q / dO stage and the S / P / dQ barrier phases
      int it = 0;
      bool ok = true;
      for (int64_t w = blockIdx.x; ok && w < n_items; w += gridDim.x, ++it) {
        const int kb = 0;
        const uint32_t aK = smem_u32(sK), aV = smem_u32(sV);
        if (!(ok = mbar_wait(&kv_full[kb], it & 1, p.status, kTimeoutMma, abort_flag))) break;
        // S^T / dP^T of block g+1 are issued as soon as the softmax warps have read block
        // g's (s_free), so they run on the tensor core while block g's P / dS are formed
        auto issue_s = [&](int64_t g) -> bool {
          const int s = static_cast<int>(g & 1);
          if (!mbar_wait(&qd_full[s], (g >> 1) & 1, p.status, kTimeoutMma, abort_flag)) return false;
          if (g >= 1 && !mbar_wait(s_free, (g - 1) & 1, p.status, kTimeoutMma, abort_flag)) return false;
          tc_fence_after();
          const uint32_t aQ = smem_u32(sQ + s * kTile), aDO = smem_u32(sDO + s * kTile);
#pragma unroll
          for (int k = 0; k < kD / 16; ++k) {
            umma_bf16_ss(tS, umma_desc_kmajor_sw128(aK + k * 32), umma_desc_kmajor_sw128(aQ + k * 32), id_s, k > 0);
            umma_bf16_ss(tDP, umma_desc_kmajor_sw128(aV + k * 32), umma_desc_kmajor_sw128(aDO + k * 32), id_s, k > 0);
          }
          umma_commit(s_full);
          return true;
        };
        if (!(ok = issue_s(gq))) break;
        // the previous item's dK / dV must have been read before block 0 overwrites them
        if (it >= 1 && !(ok = mbar_wait(acc_free, (it - 1) & 1, p.status, kTimeoutMma, abort_flag))) break;
        for (int j = 0; ok && j < n_qt; ++j, ++gq) {
          const int s = static_cast<int>(gq & 1);
          if (j + 1 < n_qt && !(ok = issue_s(gq + 1))) break;
          if (!(ok = mbar_wait(p_full, gq & 1, p.status, kTimeoutMma, abort_flag))) break;
          if (gq >= 1 && !(ok = mbar_wait(dq_free, (gq - 1) & 1, p.status, kTimeoutMma, abort_flag))) break;
          tc_fence_after();
          const uint32_t aQ = smem_u32(sQ + s * kTile), aDO = smem_u32(sDO + s * kTile);
#pragma unroll
          for (int k = 0; k < kM / 16; ++k) {
            // A = P^T from TMEM, 8 columns per 16 queries; dS^T K-major A over q: panel (k >> 2),
            // 32-byte steps; MN-major B over q rows: 2048-byte steps
            const uint64_t dS = umma_desc_kmajor_sw128(aDS + (k >> 2) * kPanel + (k & 3) * 32);
            umma_bf16_ts(tDV, tPT + k * 8, umma_smem_desc(aDO + k * 2048, 8192, 1024, 2), id_kv, (j > 0 || k > 0));
            umma_bf16_ss(tDK, dS, umma_smem_desc(aQ + k * 2048, 8192, 1024, 2), id_kv, (j > 0 || k > 0));
          }
#pragma unroll
          for (int k = 0; k < kM / 16; ++k) {
            // A = dS [q x keys] read MN-major from dS^T (rows = keys): 16 key rows per step
            const uint64_t da = umma_smem_desc(aDS + k * 2048, kPanel, 1024, 2);
            const uint64_t db = umma_smem_desc(aK + k * 2048, 8192, 1024, 2);
            umma_bf16_ss(tDQ, da, db, id_q, k > 0);
          }
          umma_commit(pds_free);
          umma_commit(dq_full);
          umma_commit(&qd_empty[s]);
        }
        if (ok) {
          umma_commit(acc_full);
          umma_commit(&kv_empty[kb]);
        }
      }
    }
  } else if (warp >= 4) {
    const int q4 = warp & 3;
    const int half = (warp - 4) >> 2;
    const int r = q4 * 32 + lane;  // TMEM lane: key row for S/dP/dK/dV, query row for dQ
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    bool ok = true;
    int64_t gq = 0;
    int it = 0;
    for (int64_t w = blockIdx.x; ok && w < n_items; w += gridDim.x, ++it) {
      int k0, i2, i1, i0;
      int64_t bh;
      item_coords(w, k0, i2, i1, i0, bh);
      const int key = k0 + r;
      const bool key_ok = key < p.Nk;
      // dQ of a block: TMEM -> this warp's 4 KB shared-memory slot (its 32 query rows x 32
      // columns, 128B-swizzled) -> one TMA tensor reduce-add into the fp32 accumulator
      uint8_t* const stg = sDQ + (warp - 4) * kDQStage;
      auto drain_dq = [&](int64_t g, int jj) -> bool {
        if (!mbar_wait_warp(dq_full, g & 1, p.status, kTimeoutEpilogue, abort_flag)) return false;
        tc_fence_after();
        uint32_t v[32];
        tmem_ld32(tDQ + lane_off + half * 32, v);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(dq_free);
          bulk_wait_read0();  // the slot's previous reduce has read it
        }
        __syncwarp();
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<float4*>(stg + lane * 128 + ((c ^ (lane & 7)) << 4)) =
              make_float4(__uint_as_float(v[4 * c]) * p.scale, __uint_as_float(v[4 * c + 1]) * p.scale,
                          __uint_as_float(v[4 * c + 2]) * p.scale, __uint_as_float(v[4 * c + 3]) * p.scale);
        fence_proxy_async_smem();
        __syncwarp();
        const int row0 = jj * kM + q4 * 32;
        if (lane == 0 && row0 < p.Nq && half * 32 < p.d_valid) {
          int c5[5];
          coords_for(p.dq_pos, row0, i2, i1, i0, c5);
          c5[0] = half * 32;
          tma_reduce_add_5d(&tmDQ, stg, c5);
          bulk_commit();
        }
        return true;
      };
      for (int j = 0; ok && j < n_qt; ++j, ++gq) {
        if (!mbar_wait_warp(s_full, gq & 1, p.status, kTimeoutEpilogue, abort_flag)) {
          ok = false;
          break;
        }
        // the block's LSE / Dvec were staged before qd_full completed (acquire it here too)
        if (!mbar_wait_warp(&qd_full[gq & 1], (gq >> 1) & 1, p.status, kTimeoutEpilogue, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float* sl = s_lse[gq & 1] + half * 64;
        const float* sd = s_dv[gq & 1] + half * 64;
        uint32_t sv[64], dp[64];
        tmem_ld32(tS + lane_off + half * 64, *reinterpret_cast<uint32_t(*)[32]>(sv));
        tmem_ld32(tS + lane_off + half * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(sv + 32));
        tmem_ld32(tDP + lane_off + half * 64, *reinterpret_cast<uint32_t(*)[32]>(dp));
        tmem_ld32(tDP + lane_off + half * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(dp + 32));
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_free);
        // P and dS of the previous block must have been consumed before we overwrite them
        if (gq >= 1 && !mbar_wait_warp(pds_free, (gq - 1) & 1, p.status, kTimeoutEpilogue, abort_flag)) {
          ok = false;
          break;
        }
        const int qbase = j * kM + half * 64;
        const uint32_t tPw = tPT + lane_off + half * 32;  // this warp's 64 queries: 32 columns
        uint8_t* panelS = sDS + half * kPanel;
        // the branch is warp-uniform: both paths end in tcgen05.st (a warp-collective store
        // that every lane must execute together), so a warp whose key rows straddle Nk takes
        // the per-element path as a whole
        if (__all_sync(0xffffffffu, key_ok && qbase + 64 <= p.Nq)) {
          // every column valid: scaling, the polynomial 2^x (half of the columns; the other
          // half on the MUFU) and dS = P (dP - D) as packed f32x2
          const uint64_t sc2 = f2pack(p.scale_log2, p.scale_log2);
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) {
            uint32_t pk[4], dk4[4];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int c0 = ch * 8 + h * 4;
              const float2 la = *reinterpret_cast<const float2*>(sl + c0);
              const float2 lb = *reinterpret_cast<const float2*>(sl + c0 + 2);
              const float2 da = *reinterpret_cast<const float2*>(sd + c0);
              const float2 db = *reinterpret_cast<const float2*>(sd + c0 + 2);
              const uint64_t xa = f2fma(f2pack(__uint_as_float(sv[c0]), __uint_as_float(sv[c0 + 1])), sc2,
                                        f2pack(la.x, la.y));
              const uint64_t xb = f2fma(f2pack(__uint_as_float(sv[c0 + 2]), __uint_as_float(sv[c0 + 3])), sc2,
                                        f2pack(lb.x, lb.y));
              float xa0, xa1, p2, p3;
              f2unpack(xa, xa0, xa1);
              const float p0 = exp2_mufu(xa0), p1 = exp2_mufu(xa1);
              exp2_poly2(xb, p2, p3);
              const uint64_t pa = f2pack(p0, p1), pb = f2pack(p2, p3);
              const uint64_t dsa =
                  f2mul(pa, f2sub(f2pack(__uint_as_float(dp[c0]), __uint_as_float(dp[c0 + 1])), f2pack(da.x, da.y)));
              const uint64_t dsb = f2mul(
                  pb, f2sub(f2pack(__uint_as_float(dp[c0 + 2]), __uint_as_float(dp[c0 + 3])), f2pack(db.x, db.y)));
              float d0, d1, d2, d3;
              f2unpack(dsa, d0, d1);
              f2unpack(dsb, d2, d3);
              pk[2 * h] = pack_bf16x2(p0, p1);
              pk[2 * h + 1] = pack_bf16x2(p2, p3);
              dk4[2 * h] = pack_bf16x2(d0, d1);
              dk4[2 * h + 1] = pack_bf16x2(d2, d3);
            }
            tmem_st4(tPw + ch * 4, pk[0], pk[1], pk[2], pk[3]);
            *reinterpret_cast<uint4*>(panelS + r * 128 + ((ch ^ (r & 7)) << 4)) =
                make_uint4(dk4[0], dk4[1], dk4[2], dk4[3]);
          }
        } else {
  #pragma unroll
          for (int ch = 0; ch < 8; ++ch) {
            uint32_t pk[4], dk4[4];
  #pragma unroll
            for (int i2p = 0; i2p < 4; ++i2p) {
              float pe[2], de[2];
  #pragma unroll
              for (int e = 0; e < 2; ++e) {
                const int col = ch * 8 + i2p * 2 + e;
                const int qi = qbase + col;
                float pv = 0.f, ds = 0.f;
                if (key_ok && qi < p.Nq) {
                  pv = exp2_mufu(fmaf(__uint_as_float(sv[col]), p.scale_log2, sl[col]));
                  ds = pv * (__uint_as_float(dp[col]) - sd[col]);
                }
                pe[e] = pv;
                de[e] = ds;
              }
              pk[i2p] = pack_bf16x2(pe[0], pe[1]);
              dk4[i2p] = pack_bf16x2(de[0], de[1]);
            }
            tmem_st4(tPw + ch * 4, pk[0], pk[1], pk[2], pk[3]);
            *reinterpret_cast<uint4*>(panelS + r * 128 + ((ch ^ (r & 7)) << 4)) =
                make_uint4(dk4[0], dk4[1], dk4[2], dk4[3]);
          }
        }
        fence_proxy_async_smem();
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
        if (j >= 1 && !drain_dq(gq - 1, j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok) ok = drain_dq(gq - 1, n_qt - 1);
      if (ok) ok = mbar_wait_warp(acc_full, it & 1, p.status, kTimeoutEpilogue, abort_flag);
      if (ok) {
        tc_fence_after();
        uint32_t v[32], wv[32];
        tmem_ld32(tDK + lane_off + half * 32, v);
        tmem_ld32(tDV + lane_off + half * 32, wv);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_free);  // the next item may overwrite dK / dV
        if (key_ok) {
          const int64_t off = static_cast<int64_t>(i0) * p.kv_s0 + static_cast<int64_t>(i1) * p.kv_s1 +
                              static_cast<int64_t>(i2) * p.kv_s2 + static_cast<int64_t>(key) * p.kv_row + half * 32;
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            if (half * 32 + c8 * 8 >= p.d_valid) continue;
            uint4 a, b;
            a.x = pack_bf16x2(__uint_as_float(v[c8 * 8]) * p.scale, __uint_as_float(v[c8 * 8 + 1]) * p.scale);
            a.y = pack_bf16x2(__uint_as_float(v[c8 * 8 + 2]) * p.scale, __uint_as_float(v[c8 * 8 + 3]) * p.scale);
            a.z = pack_bf16x2(__uint_as_float(v[c8 * 8 + 4]) * p.scale, __uint_as_float(v[c8 * 8 + 5]) * p.scale);
            a.w = pack_bf16x2(__uint_as_float(v[c8 * 8 + 6]) * p.scale, __uint_as_float(v[c8 * 8 + 7]) * p.scale);
            b.x = pack_bf16x2(__uint_as_float(wv[c8 * 8]), __uint_as_float(wv[c8 * 8 + 1]));
            b.y = pack_bf16x2(__uint_as_float(wv[c8 * 8 + 2]), __uint_as_float(wv[c8 * 8 + 3]));
            b.z = pack_bf16x2(__uint_as_float(wv[c8 * 8 + 4]), __uint_as_float(wv[c8 * 8 + 5]));
            b.w = pack_bf16x2(__uint_as_float(wv[c8 * 8 + 6]), __uint_as_float(wv[c8 * 8 + 7]));
            *reinterpret_cast<uint4*>(p.dk + off + c8 * 8) = a;
            *reinterpret_cast<uint4*>(p.dv + off + c8 * 8) = b;
          }
        }
      }
    }
  }

  if (warp >= 4 && lane == 0) bulk_wait0();  // this warp's dQ reduces have completed
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------ host

void attn_fwd_tc(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, torch::Tensor& o,
                 const c10::optional<torch::Tensor>& lse, std::vector<int64_t> lq, std::vector<int64_t> lk,
                 std::vector<int64_t> lv, std::vector<int64_t> lo, int64_t BH, int64_t Nq, int64_t Nk, int64_t d_valid,
                 double scale, const torch::Tensor& status) {
  for (const torch::Tensor* t : std::initializer_list<const torch::Tensor*>{&q, &k, &v, &o})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16, "attn_fwd_tc: bf16 CUDA tensors");
  TORCH_CHECK(d_valid > 0 && d_valid <= fa::kD && d_valid % 8 == 0, "attn_fwd_tc: head dim multiple of 8, <= 64");
  TORCH_CHECK(lk == lv || (lk[4] == lv[4] && lk[5] == lv[5]), "attn_fwd_tc: K and V share the head decomposition");
  TORCH_CHECK(lq[4] == lk[4] && lq[5] == lk[5] && lq[4] == lo[4] && lq[5] == lo[5],
              "attn_fwd_tc: Q / K / V / O share the head decomposition");
  for (int i = 0; i < 4; ++i) TORCH_CHECK(lo[i] % 8 == 0, "attn_fwd_tc: output rows must be 16-byte aligned");
  const at::cuda::CUDAGuard guard(q.device());
  if (BH == 0 || Nq == 0) return;
  TORCH_CHECK(Nk > 0, "attn_fwd_tc: at least one key");
  const int64_t n_i0 = BH / (lq[4] * lq[5]);
  TORCH_CHECK(n_i0 * lq[4] * lq[5] == BH, "attn_fwd_tc: BH must equal i0 * d1 * d2");
  Map5 mq = make_map(q, lq, Nq, n_i0, static_cast<int>(d_valid));
  Map5 mk = make_map(k, lk, Nk, n_i0, static_cast<int>(d_valid));
  Map5 mv = make_map(v, lv, Nk, n_i0, static_cast<int>(d_valid));
  TORCH_CHECK(std::equal(mk.pos, mk.pos + 4, mv.pos), "attn_fwd_tc: K and V layouts must sort alike");
  AttnTcParams p{};
  p.Nq = static_cast<int>(Nq);
  p.Nk = static_cast<int>(Nk);
  p.d_valid = static_cast<int>(d_valid);
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  std::copy(mq.pos, mq.pos + 4, p.q_pos);
  std::copy(mk.pos, mk.pos + 4, p.kv_pos);
  p.d1 = static_cast<int>(lq[4]);
  p.d2 = static_cast<int>(lq[5]);
  p.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.o_s0 = lo[0];
  p.o_s1 = lo[1];
  p.o_s2 = lo[2];
  p.o_row = lo[3];
  if (lse.has_value() && lse->defined()) {
    TORCH_CHECK(lse->scalar_type() == at::kFloat && lse->numel() >= BH * Nq, "attn_fwd_tc: fp32 lse [BH, Nq]");
    p.lse = lse->data_ptr<float>();
  }
  p.status = status.defined() && status.numel() > 0 ? status.data_ptr<int>() : nullptr;
  static bool configured[64] = {false};
  const int dev = q.get_device();
  if (!configured[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, fa::kSmemBytes));
    configured[dev] = true;
  }
  TORCH_CHECK(BH <= 2147483647LL, "attn_fwd_tc: too many heads");
  p.n_tiles_q = static_cast<int>((Nq + fa::kM - 1) / fa::kM);
  p.n_items = BH * p.n_tiles_q;
  static int n_sm[64] = {0};
  if (n_sm[dev] == 0) C10_CUDA_CHECK(cudaDeviceGetAttribute(&n_sm[dev], cudaDevAttrMultiProcessorCount, dev));
  // persistent: one CTA per SM, each looping over work items
  dim3 grid(static_cast<unsigned>(std::min<int64_t>(p.n_items, persistent_sms(n_sm[dev]))));
  attn_fwd_tc_kernel<<<grid, fa::kThreads, fa::kSmemBytes, at::cuda::getCurrentCUDAStream()>>>(mq.map, mk.map, mv.map, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// dK / dV share one layout (ldkv); dq is a zeroed fp32 accumulator addressed through ldq
// (same head decomposition; 8-byte aligned rows)
void attn_bwd_tc(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, const torch::Tensor& dout,
                 const torch::Tensor& lse, const torch::Tensor& dvec, torch::Tensor& dq, torch::Tensor& dk,
                 torch::Tensor& dv, std::vector<int64_t> lq, std::vector<int64_t> lkv, std::vector<int64_t> ldo,
                 std::vector<int64_t> ldkv, std::vector<int64_t> ldq, int64_t BH, int64_t Nq, int64_t Nk,
                 int64_t d_valid, double scale, const torch::Tensor& status) {
  for (const torch::Tensor* t : std::initializer_list<const torch::Tensor*>{&q, &k, &v, &dout, &dk, &dv})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16, "attn_bwd_tc: bf16 CUDA tensors");
  TORCH_CHECK(dq.is_cuda() && dq.scalar_type() == at::kFloat, "attn_bwd_tc: dq must be a zeroed fp32 accumulator");
  for (int i = 0; i < 4; ++i)
    TORCH_CHECK(ldq[i] % 4 == 0, "attn_bwd_tc: dq accumulator strides must be multiples of 4 (16-byte TMA reduce)");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && dvec.scalar_type() == at::kFloat, "attn_bwd_tc: fp32 lse / dvec");
  TORCH_CHECK(d_valid > 0 && d_valid <= 64 && d_valid % 8 == 0, "attn_bwd_tc: head dim multiple of 8, <= 64");
  TORCH_CHECK(lq[4] == lkv[4] && lq[5] == lkv[5] && lq[4] == ldo[4] && lq[5] == ldo[5] && lq[4] == ldkv[4] &&
                  lq[5] == ldkv[5],
              "attn_bwd_tc: shared head decomposition");
  for (int i = 0; i < 4; ++i) TORCH_CHECK(ldkv[i] % 8 == 0, "attn_bwd_tc: dK / dV rows must be 16-byte aligned");
  const at::cuda::CUDAGuard guard(q.device());
  if (BH == 0 || Nq == 0 || Nk == 0) return;
  const int64_t n_i0 = BH / (lq[4] * lq[5]);
  Map5 mq = make_map(q, lq, Nq, n_i0, static_cast<int>(d_valid));
  Map5 mdo = make_map(dout, ldo, Nq, n_i0, static_cast<int>(d_valid));
  Map5 mk = make_map(k, lkv, Nk, n_i0, static_cast<int>(d_valid));
  Map5 mv = make_map(v, lkv, Nk, n_i0, static_cast<int>(d_valid));
  // fp32 dQ accumulator: 32-column x 32-row boxes (one drain warp's slot), 128B-swizzled
  Map5 mdq = make_map(dq, ldq, Nq, n_i0, static_cast<int>(d_valid), 4, 32, 32, CU_TENSOR_MAP_DATA_TYPE_FLOAT32);
  TORCH_CHECK(std::equal(mq.pos, mq.pos + 4, mdo.pos), "attn_bwd_tc: Q and dO layouts must sort alike");
  AttnBwdTcParams p{};
  p.Nq = static_cast<int>(Nq);
  p.Nk = static_cast<int>(Nk);
  p.d_valid = static_cast<int>(d_valid);
  p.scale = static_cast<float>(scale);
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  std::copy(mq.pos, mq.pos + 4, p.q_pos);
  std::copy(mk.pos, mk.pos + 4, p.kv_pos);
  std::copy(mdq.pos, mdq.pos + 4, p.dq_pos);
  p.d1 = static_cast<int>(lq[4]);
  p.d2 = static_cast<int>(lq[5]);
  p.lse = lse.data_ptr<float>();
  p.dvec = dvec.data_ptr<float>();
  p.dq = dq.data_ptr<float>();
  p.dq_s0 = ldq[0];
  p.dq_s1 = ldq[1];
  p.dq_s2 = ldq[2];
  p.dq_row = ldq[3];
  p.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  p.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  p.kv_s0 = ldkv[0];
  p.kv_s1 = ldkv[1];
  p.kv_s2 = ldkv[2];
  p.kv_row = ldkv[3];
  p.status = status.defined() && status.numel() > 0 ? status.data_ptr<int>() : nullptr;
  p.n_tiles_k = static_cast<int>((Nk + fb::kM - 1) / fb::kM);
  static bool configured[64] = {false};
  const int dev = q.get_device();
  if (!configured[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, fb::kSmemBytes));
    configured[dev] = true;
  }
  p.n_items = BH * p.n_tiles_k;
  static int n_sm[64] = {0};
  if (n_sm[dev] == 0) C10_CUDA_CHECK(cudaDeviceGetAttribute(&n_sm[dev], cudaDevAttrMultiProcessorCount, dev));
  // persistent: one CTA per SM, each looping over (head, key tile) work items
  attn_bwd_tc_kernel<<<static_cast<unsigned>(std::min<int64_t>(p.n_items, persistent_sms(n_sm[dev]))), fb::kThreads, fb::kSmemBytes,
                       at::cuda::getCurrentCUDAStream()>>>(mq.map, mk.map, mv.map, mdo.map, mdq.map, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Element-wise exp2_poly over a tensor: lets the tests check the softmax's FMA-pipe
// exponential against CUDA's exp2f over its whole input range.
__global__ void exp2_poly_eval_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) y[i] = exp2_poly(x[i]);
}

torch::Tensor exp2_poly_eval(const torch::Tensor& x) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat && x.is_contiguous(), "exp2_poly_eval: fp32 CUDA tensor");
  const at::cuda::CUDAGuard guard(x.device());
  auto y = torch::empty_like(x);
  const int64_t n = x.numel();
  if (n == 0) return y;
  exp2_poly_eval_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      x.data_ptr<float>(), y.data_ptr<float>(), n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return y;
}

}  // namespace nori
