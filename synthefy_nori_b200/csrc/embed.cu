// Feature-embedding kernels of the Nori input side (training and inference).
//
// K1  col_stats          one pass set per (table, feature column) over the context rows:
//                        finite mean (NaN / inf fill value), standard deviation of the
//                        filled column (unbiased, +1e-20 guard), and whether the column
//                        is usable (>1 finite value, min != max); then, per feature
//                        group, the sqrt(fpg / n_valid) rescale; per table the finite
//                        mean of the context targets (y NaN fill).
// K2  rbf_aug_fwd/bwd    per token (one table row x one feature group): the preprocessed
//                        value of each cell (fill, standardise, clip +-100, group
//                        rescale), its scientific decomposition |v| = m 10^e (in fp64),
//                        64 Gaussian kernels on m, the (sign, exponent) gate, LayerNorm;
//                        the row written for the fused embedding GEMM is
//                        [r_0 (64), present_0, missing_0, r_1 (64), present_1, missing_1,
//                        0 pad]: the per-cell Linear (64 -> E) and the first fusion
//                        Linear (fpg E -> E) have no nonlinearity between them, so the
//                        caller multiplies this row by their precomposed weights (one
//                        GEMM with K = 136 instead of a [cells, E] intermediate and a
//                        K = fpg E GEMM); the two indicator columns carry the out-layer
//                        bias (present) and the learned missing-cell vector (missing).
//                        The backward recomputes the forward per token and accumulates
//                        the gate-table and LayerNorm gradients (one warp per token,
//                        lane k owns kernels k and k + 32, so the table updates of a
//                        warp never collide).
// K3  assemble_fwd/bwd   per table row: the target-aware gate on every feature token
//                        (x + (1 - a) rb + a rb sigmoid(x . rb / sqrt(E)), rb = w y + b
//                        from the context target; query rows unchanged), the y token
//                        (Linear(2 -> E) of the filled target and its NaN indicator), all
//                        written straight into the encoder's token-row matrix (context
//                        rows first, then query rows, G + 1 tokens per table row).
//
// Reference: model/encoders.py:12-77 (statistics), 588-653 (NaN), 656-724 (valid
// features), 118-276 (scientific RBF), 432-585 (mask embedding + fusion), 727-969 (y
// encoders); model/transformer.py:1080-1132 (target-aware embedding).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>

#include "sm100.cuh"

namespace nori {

constexpr int kRbfK = 64;       // Gaussian kernels per cell
constexpr int kRbfTable = 38;   // (sign, exponent in [-9, 9]) control tokens
constexpr int kMaxExp = 9;

// ------------------------------------------------------------------ K1
// grid (B, ceil(F / 32)); 8 warps; lane = feature within the 32-wide chunk, warps split
// the context rows.  Outputs per (b, f): mean [B, F], stdv [B, F]; per (b, g):
// gscale [B, G]; per b: ymean [B] (chunk 0 of each table).
__global__ void col_stats_kernel(const float* __restrict__ x, int S, int F, int ep, int fpg,
                                 const float* __restrict__ y, int ylen, float* __restrict__ mean_out,
                                 float* __restrict__ std_out, float* __restrict__ gscale_out,
                                 float* __restrict__ ymean_out, int* __restrict__ nvalid_out) {
  const int b = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
  const int f = blockIdx.y * 32 + lane;
  const bool live = f < F;
  const float* xb = x + static_cast<int64_t>(b) * S * F;
  __shared__ float s_sum[8][32], s_cnt[8][32], s_min[8][32], s_max[8][32], s_sq[8][32];
  float sum = 0.f, cnt = 0.f, mn = INFINITY, mx = -INFINITY;
  if (live) {
    for (int r = warp; r < ep; r += warps) {
      const float v = xb[static_cast<int64_t>(r) * F + f];
      if (isfinite(v)) {
        sum += v;
        cnt += 1.f;
        mn = fminf(mn, v);
        mx = fmaxf(mx, v);
      }
    }
  }
  s_sum[warp][lane] = sum;
  s_cnt[warp][lane] = cnt;
  s_min[warp][lane] = mn;
  s_max[warp][lane] = mx;
  __syncthreads();
  float tsum = 0.f, tcnt = 0.f, tmn = INFINITY, tmx = -INFINITY;
  for (int w = 0; w < warps; ++w) {
    tsum += s_sum[w][lane];
    tcnt += s_cnt[w][lane];
    tmn = fminf(tmn, s_min[w][lane]);
    tmx = fmaxf(tmx, s_max[w][lane]);
  }
  const float mean = tsum / fmaxf(tcnt, 1.f);  // fill value == mean of the filled column
  float sq = 0.f;
  if (live) {
    for (int r = warp; r < ep; r += warps) {
      const float v = xb[static_cast<int64_t>(r) * F + f];
      if (isfinite(v)) {
        const float d = mean - v;
        sq += d * d;
      }
    }
  }
  s_sq[warp][lane] = sq;
  __syncthreads();
  float tsq = 0.f;
  for (int w = 0; w < warps; ++w) tsq += s_sq[w][lane];
  float stdv = sqrtf(tsq / static_cast<float>(max(ep - 1, 1))) + 1e-20f;
  if (S == 1 || ep == 1) stdv = 1.f;
  // usable column: >1 finite value and min != max after standardisation and the +-100
  // clip (both monotone, so the transformed extremes are the transformed raw extremes)
  const float zmn = fminf(fmaxf((tmn - mean) / stdv, -100.f), 100.f);
  const float zmx = fminf(fmaxf((tmx - mean) / stdv, -100.f), 100.f);
  const bool valid = live && tcnt > 1.f && zmn != zmx;
  // group counts: fpg divides 32, so a group's features sit in consecutive lanes
  int nv = valid ? 1 : 0;
  for (int o = 1; o < fpg; o <<= 1) nv += __shfl_xor_sync(0xffffffffu, nv, o);
  if (warp == 0 && live) {
    mean_out[static_cast<int64_t>(b) * F + f] = mean;
    std_out[static_cast<int64_t>(b) * F + f] = stdv;
    if ((f % fpg) == 0) {
      const int G = F / fpg;
      const int nvc = max(nv, 1);
      gscale_out[static_cast<int64_t>(b) * G + f / fpg] = sqrtf(static_cast<float>(fpg) / static_cast<float>(nvc));
      nvalid_out[static_cast<int64_t>(b) * G + f / fpg] = nvc;
    }
  }
  if (blockIdx.y == 0 && warp == 0 && y != nullptr) {  // y: finite mean over the context rows
    float ys = 0.f, yc = 0.f;
    for (int r = lane; r < ep; r += 32) {
      const float v = y[static_cast<int64_t>(b) * ylen + r];
      if (isfinite(v)) {
        ys += v;
        yc += 1.f;
      }
    }
    ys = warp_sum(ys);
    yc = warp_sum(yc);
    if (lane == 0) ymean_out[b] = ys / fmaxf(yc, 1.f);
  }
}

// ------------------------------------------------------------------ K2
struct RbfArgs {
  const float* x;       // raw [B, S, F]
  const float* mean;    // [B, F]
  const float* stdv;    // [B, F]
  const float* gscale;  // [B, G]
  const float* table;   // [38, 128]: gamma (64) | beta (64), activations applied
  const float* ln_w;    // [64]
  const float* ln_b;    // [64]
  const float* centers; // [64]
  double inv_two_sigma2;
  float ln_eps;
  int B, S, F, G, fpg, kaug;
};

// Preprocessed value of cell (b, s, f): NaN for missing (non-finite raw) cells.
__device__ __forceinline__ float prep_value(const RbfArgs& a, int b, int s, int f) {
  const float v = a.x[(static_cast<int64_t>(b) * a.S + s) * a.F + f];
  if (!isfinite(v)) return NAN;
  const float m = a.mean[static_cast<int64_t>(b) * a.F + f];
  float z = (v - m) / a.stdv[static_cast<int64_t>(b) * a.F + f];
  z = fminf(fmaxf(z, -100.f), 100.f);
  return z * a.gscale[static_cast<int64_t>(b) * a.G + f / a.fpg];
}

// |v| = m 10^e, e = clamp(floor(log10 |v|), -9, 9), in fp64; table row of (sign, e).
__device__ __forceinline__ void decompose(float v, double& m, int& row) {
  const double av = fabs(static_cast<double>(v));
  int e = 0;
  if (av > 0.0) {
    e = static_cast<int>(floor(log10(av)));
    e = e < -kMaxExp ? -kMaxExp : (e > kMaxExp ? kMaxExp : e);
    m = av / exp10(static_cast<double>(e));
  } else {
    m = 0.0;
  }
  row = (v < 0.f ? 1 : 0) * (2 * kMaxExp + 1) + (e + kMaxExp);
}

// One warp per token; lane owns kernels lane and lane + 32 of each cell.
__global__ void rbf_aug_fwd_kernel(RbfArgs a, int64_t n_tokens, __nv_bfloat16* __restrict__ out) {
  __shared__ float s_tab[kRbfTable * 2 * kRbfK];
  for (int i = threadIdx.x; i < kRbfTable * 2 * kRbfK; i += blockDim.x) s_tab[i] = a.table[i];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const float c0 = a.centers[lane], c1 = a.centers[lane + 32];
  const float w0 = a.ln_w[lane], w1 = a.ln_w[lane + 32], bb0 = a.ln_b[lane], bb1 = a.ln_b[lane + 32];
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * warps + (threadIdx.x >> 5); t < n_tokens;
       t += static_cast<int64_t>(gridDim.x) * warps) {
    const int g = static_cast<int>(t % a.G);
    const int64_t bs = t / a.G;
    const int s = static_cast<int>(bs % a.S), b = static_cast<int>(bs / a.S);
    __nv_bfloat16* o = out + t * a.kaug;
    for (int c = 0; c < a.fpg; ++c) {
      const float v = prep_value(a, b, s, g * a.fpg + c);
      __nv_bfloat16* oc = o + c * (kRbfK + 2);
      if (!isfinite(v)) {  // missing cell: r = 0, missing indicator
        oc[lane] = __float2bfloat16(0.f);
        oc[lane + 32] = __float2bfloat16(0.f);
        if (lane == 0) {
          oc[kRbfK] = __float2bfloat16(0.f);
          oc[kRbfK + 1] = __float2bfloat16(1.f);
        }
        continue;
      }
      double m;
      int row;
      decompose(v, m, row);
      const double d0 = m - static_cast<double>(c0), d1 = m - static_cast<double>(c1);
      const float r0 = static_cast<float>(exp(-(d0 * d0) * a.inv_two_sigma2));
      const float r1 = static_cast<float>(exp(-(d1 * d1) * a.inv_two_sigma2));
      const float* tr = s_tab + row * 2 * kRbfK;
      const float z0 = r0 * tr[lane] + tr[kRbfK + lane];
      const float z1 = r1 * tr[lane + 32] + tr[kRbfK + lane + 32];
      const float mean = warp_sum(z0 + z1) * (1.f / kRbfK);
      const float e0 = z0 - mean, e1 = z1 - mean;
      const float rstd = rsqrtf(warp_sum(e0 * e0 + e1 * e1) * (1.f / kRbfK) + a.ln_eps);
      oc[lane] = __float2bfloat16(e0 * rstd * w0 + bb0);
      oc[lane + 32] = __float2bfloat16(e1 * rstd * w1 + bb1);
      if (lane == 0) {
        oc[kRbfK] = __float2bfloat16(1.f);
        oc[kRbfK + 1] = __float2bfloat16(0.f);
      }
    }
    for (int k = a.fpg * (kRbfK + 2) + lane; k < a.kaug; k += 32) o[k] = __float2bfloat16(0.f);
  }
}

// dR [n_tokens, kaug] bf16 -> d table [38, 128], d ln_w [64], d ln_b [64] (fp32, +=).
__global__ void rbf_aug_bwd_kernel(RbfArgs a, int64_t n_tokens, const __nv_bfloat16* __restrict__ dr,
                                   float* __restrict__ dtable, float* __restrict__ dlnw, float* __restrict__ dlnb) {
  __shared__ float s_tab[kRbfTable * 2 * kRbfK];
  __shared__ float s_dtab[kRbfTable * 2 * kRbfK];
  for (int i = threadIdx.x; i < kRbfTable * 2 * kRbfK; i += blockDim.x) {
    s_tab[i] = a.table[i];
    s_dtab[i] = 0.f;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const float c0 = a.centers[lane], c1 = a.centers[lane + 32];
  const float w0 = a.ln_w[lane], w1 = a.ln_w[lane + 32];
  float gw0 = 0.f, gw1 = 0.f, gb0 = 0.f, gb1 = 0.f;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * warps + (threadIdx.x >> 5); t < n_tokens;
       t += static_cast<int64_t>(gridDim.x) * warps) {
    const int g = static_cast<int>(t % a.G);
    const int64_t bs = t / a.G;
    const int s = static_cast<int>(bs % a.S), b = static_cast<int>(bs / a.S);
    const __nv_bfloat16* drow = dr + t * a.kaug;
    for (int c = 0; c < a.fpg; ++c) {
      const float v = prep_value(a, b, s, g * a.fpg + c);
      if (!isfinite(v)) continue;
      double m;
      int row;
      decompose(v, m, row);
      const double d0 = m - static_cast<double>(c0), d1 = m - static_cast<double>(c1);
      const float r0 = static_cast<float>(exp(-(d0 * d0) * a.inv_two_sigma2));
      const float r1 = static_cast<float>(exp(-(d1 * d1) * a.inv_two_sigma2));
      const float* tr = s_tab + row * 2 * kRbfK;
      const float z0 = r0 * tr[lane] + tr[kRbfK + lane];
      const float z1 = r1 * tr[lane + 32] + tr[kRbfK + lane + 32];
      const float mean = warp_sum(z0 + z1) * (1.f / kRbfK);
      const float e0 = z0 - mean, e1 = z1 - mean;
      const float rstd = rsqrtf(warp_sum(e0 * e0 + e1 * e1) * (1.f / kRbfK) + a.ln_eps);
      const float h0 = e0 * rstd, h1 = e1 * rstd;
      const float g0 = __bfloat162float(drow[c * (kRbfK + 2) + lane]);
      const float g1 = __bfloat162float(drow[c * (kRbfK + 2) + lane + 32]);
      gw0 += g0 * h0;
      gw1 += g1 * h1;
      gb0 += g0;
      gb1 += g1;
      const float dh0 = g0 * w0, dh1 = g1 * w1;
      const float mdh = warp_sum(dh0 + dh1) * (1.f / kRbfK);
      const float mdhh = warp_sum(dh0 * h0 + dh1 * h1) * (1.f / kRbfK);
      const float dz0 = rstd * (dh0 - mdh - h0 * mdhh);
      const float dz1 = rstd * (dh1 - mdh - h1 * mdhh);
      float* dt = s_dtab + row * 2 * kRbfK;
      atomicAdd(dt + lane, dz0 * r0);
      atomicAdd(dt + lane + 32, dz1 * r1);
      atomicAdd(dt + kRbfK + lane, dz0);
      atomicAdd(dt + kRbfK + lane + 32, dz1);
    }
  }
  atomicAdd(dlnw + lane, gw0);
  atomicAdd(dlnw + lane + 32, gw1);
  atomicAdd(dlnb + lane, gb0);
  atomicAdd(dlnb + lane + 32, gb1);
  __syncthreads();
  for (int i = threadIdx.x; i < kRbfTable * 2 * kRbfK; i += blockDim.x)
    if (s_dtab[i] != 0.f) atomicAdd(dtable + i, s_dtab[i]);
}

// ------------------------------------------------------------------ K3
struct AsmArgs {
  const __nv_bfloat16* h;  // [B, S, G, E] final LayerNorm output of the fusion MLP
  const float* y;          // [B, ylen] raw targets (context part used)
  const float* ymean;      // [B]
  const float* w_ta;       // [E] target-aware Linear(1 -> E)
  const float* b_ta;       // [E]
  const float* alpha;      // [1] sigmoid(column_y_aware_alpha), device scalar (or null)
  const float* w_y;        // [E, 2] y encoder Linear(2 -> E)
  const float* b_y;        // [E]
  float inv_sqrt_e, ta_scale;
  int B, S, G, E, ep, ylen, column_gate, use_ta;
};

__device__ __forceinline__ int64_t token_row(int b, int s, int t, int B, int S, int ep, int T) {
  if (s < ep) return (static_cast<int64_t>(b) * ep + s) * T + t;
  const int64_t rctx = static_cast<int64_t>(B) * ep * T;
  return rctx + (static_cast<int64_t>(b) * (S - ep) + (s - ep)) * T + t;
}

constexpr int kAsmMaxPerLane = 16;  // E <= 512

// One warp per table row (b, s): G feature tokens + the y token.
__global__ void assemble_fwd_kernel(AsmArgs a, __nv_bfloat16* __restrict__ X) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= static_cast<int64_t>(a.B) * a.S) return;
  const int b = static_cast<int>(row / a.S), s = static_cast<int>(row % a.S);
  const int T = a.G + 1;
  const bool ctx = s < a.ep;
  const float yv = ctx ? a.y[static_cast<int64_t>(b) * a.ylen + s] : NAN;
  const float al = a.alpha != nullptr ? *a.alpha : 0.f;
  float rb[kAsmMaxPerLane];
#pragma unroll
  for (int i = 0; i < kAsmMaxPerLane; ++i) {
    const int e = lane + 32 * i;
    rb[i] = (e < a.E && ctx && a.use_ta) ? (a.w_ta[e] * yv + a.b_ta[e]) * a.ta_scale : 0.f;
  }
  for (int g = 0; g < a.G; ++g) {
    const __nv_bfloat16* hr = a.h + (row * a.G + g) * a.E;
    __nv_bfloat16* xr = X + token_row(b, s, g, a.B, a.S, a.ep, T) * a.E;
    float hv[kAsmMaxPerLane];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < kAsmMaxPerLane; ++i) {
      const int e = lane + 32 * i;
      hv[i] = e < a.E ? __bfloat162float(hr[e]) : 0.f;
      dot += hv[i] * rb[i];
    }
    float gate = 0.f;
    if (ctx && a.use_ta && a.column_gate) gate = 1.f / (1.f + __expf(-warp_sum(dot) * a.inv_sqrt_e));
#pragma unroll
    for (int i = 0; i < kAsmMaxPerLane; ++i) {
      const int e = lane + 32 * i;
      if (e < a.E) {
        float o = hv[i];
        if (ctx && a.use_ta) o += a.column_gate ? (1.f - al) * rb[i] + al * rb[i] * gate : rb[i];
        xr[e] = __float2bfloat16(o);
      }
    }
  }
  // y token: Linear(2 -> E) of (filled target, NaN indicator); query rows are masked
  const float yf = isfinite(yv) ? yv : a.ymean[b];
  const float ind = isnan(yv) ? -2.f : (isinf(yv) ? (yv > 0.f ? 2.f : 4.f) : 0.f);
  __nv_bfloat16* yr = X + token_row(b, s, a.G, a.B, a.S, a.ep, T) * a.E;
  for (int e = lane; e < a.E; e += 32) yr[e] = __float2bfloat16(a.w_y[2 * e] * yf + a.w_y[2 * e + 1] * ind + a.b_y[e]);
}

// dX [R, E] bf16 -> dh [B, S, G, E] bf16; d w_ta, d b_ta, d w_y [E, 2], d b_y [E], d alpha (fp32, +=).
__global__ void assemble_bwd_kernel(AsmArgs a, const __nv_bfloat16* __restrict__ dX, __nv_bfloat16* __restrict__ dh,
                                    float* __restrict__ dw_ta, float* __restrict__ db_ta, float* __restrict__ dw_y,
                                    float* __restrict__ db_y, float* __restrict__ dalpha) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= static_cast<int64_t>(a.B) * a.S) return;
  const int b = static_cast<int>(row / a.S), s = static_cast<int>(row % a.S);
  const int T = a.G + 1;
  const bool ctx = s < a.ep;
  const bool ta = ctx && a.use_ta;
  const float yv = ctx ? a.y[static_cast<int64_t>(b) * a.ylen + s] : NAN;
  const float al = a.alpha != nullptr ? *a.alpha : 0.f;
  float rb[kAsmMaxPerLane], drb[kAsmMaxPerLane];
#pragma unroll
  for (int i = 0; i < kAsmMaxPerLane; ++i) {
    const int e = lane + 32 * i;
    rb[i] = (e < a.E && ta) ? (a.w_ta[e] * yv + a.b_ta[e]) * a.ta_scale : 0.f;
    drb[i] = 0.f;
  }
  float dal = 0.f;
  for (int g = 0; g < a.G; ++g) {
    const __nv_bfloat16* hr = a.h + (row * a.G + g) * a.E;
    const __nv_bfloat16* dxr = dX + token_row(b, s, g, a.B, a.S, a.ep, T) * a.E;
    __nv_bfloat16* dhr = dh + (row * a.G + g) * a.E;
    if (!ta) {
      for (int e = lane; e < a.E; e += 32) dhr[e] = dxr[e];
      continue;
    }
    float hv[kAsmMaxPerLane], dv[kAsmMaxPerLane];
    float dot = 0.f, drbdot = 0.f;
#pragma unroll
    for (int i = 0; i < kAsmMaxPerLane; ++i) {
      const int e = lane + 32 * i;
      hv[i] = e < a.E ? __bfloat162float(hr[e]) : 0.f;
      dv[i] = e < a.E ? __bfloat162float(dxr[e]) : 0.f;
      dot += hv[i] * rb[i];
      drbdot += dv[i] * rb[i];
    }
    drbdot = warp_sum(drbdot);
    if (a.column_gate) {
      const float gate = 1.f / (1.f + __expf(-warp_sum(dot) * a.inv_sqrt_e));
      const float gg = al * gate * (1.f - gate) * a.inv_sqrt_e * drbdot;  // d/du of a * gate * (rb . dout)
      dal += (gate - 1.f) * drbdot;
#pragma unroll
      for (int i = 0; i < kAsmMaxPerLane; ++i) {
        const int e = lane + 32 * i;
        if (e < a.E) {
          dhr[e] = __float2bfloat16(dv[i] + gg * rb[i]);
          drb[i] += ((1.f - al) + al * gate) * dv[i] + gg * hv[i];
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < kAsmMaxPerLane; ++i) {
        const int e = lane + 32 * i;
        if (e < a.E) {
          dhr[e] = __float2bfloat16(dv[i]);
          drb[i] += dv[i];
        }
      }
    }
  }
  if (ta) {
#pragma unroll
    for (int i = 0; i < kAsmMaxPerLane; ++i) {
      const int e = lane + 32 * i;
      if (e < a.E) {
        const float d = drb[i] * a.ta_scale;
        atomicAdd(dw_ta + e, d * yv);
        atomicAdd(db_ta + e, d);
      }
    }
    if (lane == 0 && dalpha != nullptr && a.column_gate) atomicAdd(dalpha, dal);
  }
  const float yf = isfinite(yv) ? yv : a.ymean[b];
  const float ind = isnan(yv) ? -2.f : (isinf(yv) ? (yv > 0.f ? 2.f : 4.f) : 0.f);
  const __nv_bfloat16* dyr = dX + token_row(b, s, a.G, a.B, a.S, a.ep, T) * a.E;
  for (int e = lane; e < a.E; e += 32) {
    const float d = __bfloat162float(dyr[e]);
    atomicAdd(dw_y + 2 * e, d * yf);
    atomicAdd(dw_y + 2 * e + 1, d * ind);
    atomicAdd(db_y + e, d);
  }
}

// ------------------------------------------------------------------ host
static void f32c(const torch::Tensor& t, int64_t n, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kFloat && t.is_contiguous() && t.numel() == n, what,
              ": contiguous fp32 CUDA tensor of ", n, " elements expected");
}

// x [B, S, F] fp32 raw (NaN / inf allowed), y [B, ylen] fp32 or empty -> (mean [B, F],
// std [B, F], gscale [B, G], ymean [B], nvalid [B, G] int32)
std::vector<torch::Tensor> col_stats(const torch::Tensor& x, int64_t ep, int64_t fpg, const torch::Tensor& y) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat && x.is_contiguous() && x.dim() == 3,
              "col_stats: contiguous fp32 [B, S, F]");
  const int B = static_cast<int>(x.size(0)), S = static_cast<int>(x.size(1)), F = static_cast<int>(x.size(2));
  TORCH_CHECK(fpg >= 1 && fpg <= 32 && (fpg & (fpg - 1)) == 0 && F % fpg == 0,
              "col_stats: fpg a power of two <= 32 dividing F");
  TORCH_CHECK(ep >= 1 && ep <= S, "col_stats: 1 <= eval_pos <= S");
  const at::cuda::CUDAGuard guard(x.device());
  const int G = F / static_cast<int>(fpg);
  auto o = x.options();
  auto mean = torch::empty({B, F}, o), stdv = torch::empty({B, F}, o), gs = torch::empty({B, G}, o);
  auto ym = torch::zeros({B}, o);
  auto nv = torch::empty({B, G}, o.dtype(at::kInt));
  const float* yp = nullptr;
  int ylen = 0;
  if (y.defined() && y.numel() > 0) {
    TORCH_CHECK(y.scalar_type() == at::kFloat && y.is_contiguous() && y.dim() == 2 && y.size(0) == B &&
                    y.size(1) >= ep,
                "col_stats: fp32 y [B, >= ep]");
    yp = y.data_ptr<float>();
    ylen = static_cast<int>(y.size(1));
  }
  if (B == 0) return {mean, stdv, gs, ym, nv};
  const dim3 grid(B, (F + 31) / 32);
  col_stats_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      x.data_ptr<float>(), S, F, static_cast<int>(ep), static_cast<int>(fpg), yp, ylen, mean.data_ptr<float>(),
      stdv.data_ptr<float>(), gs.data_ptr<float>(), ym.data_ptr<float>(), nv.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {mean, stdv, gs, ym, nv};
}

static RbfArgs rbf_args(const torch::Tensor& x, const torch::Tensor& mean, const torch::Tensor& stdv,
                        const torch::Tensor& gscale, const torch::Tensor& table, const torch::Tensor& ln_w,
                        const torch::Tensor& ln_b, const torch::Tensor& centers, double sigma, double ln_eps,
                        int64_t fpg, int64_t kaug) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat && x.is_contiguous() && x.dim() == 3,
              "rbf_aug: contiguous fp32 x [B, S, F]");
  const int B = static_cast<int>(x.size(0)), S = static_cast<int>(x.size(1)), F = static_cast<int>(x.size(2));
  TORCH_CHECK(fpg >= 1 && F % fpg == 0, "rbf_aug: F a multiple of fpg");
  const int G = F / static_cast<int>(fpg);
  f32c(mean, static_cast<int64_t>(B) * F, "mean");
  f32c(stdv, static_cast<int64_t>(B) * F, "std");
  f32c(gscale, static_cast<int64_t>(B) * G, "gscale");
  f32c(table, kRbfTable * 2 * kRbfK, "gate table [38, 128]");
  f32c(ln_w, kRbfK, "ln_w");
  f32c(ln_b, kRbfK, "ln_b");
  f32c(centers, kRbfK, "centers");
  TORCH_CHECK(kaug >= fpg * (kRbfK + 2) && kaug % 8 == 0, "rbf_aug: kaug >= fpg * 66, a multiple of 8");
  TORCH_CHECK(sigma > 0.0, "rbf_aug: positive sigma");
  RbfArgs a;
  a.x = x.data_ptr<float>();
  a.mean = mean.data_ptr<float>();
  a.stdv = stdv.data_ptr<float>();
  a.gscale = gscale.data_ptr<float>();
  a.table = table.data_ptr<float>();
  a.ln_w = ln_w.data_ptr<float>();
  a.ln_b = ln_b.data_ptr<float>();
  a.centers = centers.data_ptr<float>();
  a.inv_two_sigma2 = 1.0 / (2.0 * sigma * sigma);
  a.ln_eps = static_cast<float>(ln_eps);
  a.B = B;
  a.S = S;
  a.F = F;
  a.G = G;
  a.fpg = static_cast<int>(fpg);
  a.kaug = static_cast<int>(kaug);
  return a;
}

static unsigned warp_grid(int64_t items, int dev) {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((items + 7) / 8, 8 * std::max(sms, 1))));
}

torch::Tensor rbf_aug_fwd(const torch::Tensor& x, const torch::Tensor& mean, const torch::Tensor& stdv,
                          const torch::Tensor& gscale, const torch::Tensor& table, const torch::Tensor& ln_w,
                          const torch::Tensor& ln_b, const torch::Tensor& centers, double sigma, double ln_eps,
                          int64_t fpg, int64_t kaug) {
  RbfArgs a = rbf_args(x, mean, stdv, gscale, table, ln_w, ln_b, centers, sigma, ln_eps, fpg, kaug);
  const at::cuda::CUDAGuard guard(x.device());
  const int64_t n = static_cast<int64_t>(a.B) * a.S * a.G;
  auto out = torch::empty({n, kaug}, x.options().dtype(at::kBFloat16));
  if (n == 0) return out;
  rbf_aug_fwd_kernel<<<warp_grid(n, x.get_device()), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      a, n, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

void rbf_aug_bwd(const torch::Tensor& x, const torch::Tensor& mean, const torch::Tensor& stdv,
                 const torch::Tensor& gscale, const torch::Tensor& table, const torch::Tensor& ln_w,
                 const torch::Tensor& ln_b, const torch::Tensor& centers, double sigma, double ln_eps, int64_t fpg,
                 const torch::Tensor& dr, torch::Tensor& dtable, torch::Tensor& dlnw, torch::Tensor& dlnb) {
  TORCH_CHECK(dr.is_cuda() && dr.scalar_type() == at::kBFloat16 && dr.is_contiguous() && dr.dim() == 2,
              "rbf_aug_bwd: contiguous bf16 dR");
  RbfArgs a = rbf_args(x, mean, stdv, gscale, table, ln_w, ln_b, centers, sigma, ln_eps, fpg, dr.size(1));
  const int64_t n = static_cast<int64_t>(a.B) * a.S * a.G;
  TORCH_CHECK(dr.size(0) == n, "rbf_aug_bwd: one dR row per token");
  f32c(dtable, kRbfTable * 2 * kRbfK, "dtable");
  f32c(dlnw, kRbfK, "dlnw");
  f32c(dlnb, kRbfK, "dlnb");
  const at::cuda::CUDAGuard guard(x.device());
  if (n == 0) return;
  rbf_aug_bwd_kernel<<<warp_grid(n, x.get_device()), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      a, n, reinterpret_cast<const __nv_bfloat16*>(dr.data_ptr()), dtable.data_ptr<float>(), dlnw.data_ptr<float>(),
      dlnb.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static AsmArgs asm_args(const torch::Tensor& h, const torch::Tensor& y, const torch::Tensor& ymean,
                        const c10::optional<torch::Tensor>& w_ta, const c10::optional<torch::Tensor>& b_ta,
                        const c10::optional<torch::Tensor>& alpha, const torch::Tensor& w_y, const torch::Tensor& b_y,
                        int64_t B, int64_t S, int64_t G, int64_t ep, double ta_scale) {
  TORCH_CHECK(h.is_cuda() && h.scalar_type() == at::kBFloat16 && h.is_contiguous() && h.dim() == 2 &&
                  h.size(0) == B * S * G,
              "assemble: contiguous bf16 h [B * S * G, E]");
  const int E = static_cast<int>(h.size(1));
  TORCH_CHECK(E <= 32 * kAsmMaxPerLane, "assemble: E <= 512");
  TORCH_CHECK(y.is_cuda() && y.scalar_type() == at::kFloat && y.is_contiguous() && y.dim() == 2 && y.size(0) == B &&
                  y.size(1) >= ep,
              "assemble: fp32 y [B, >= ep]");
  f32c(ymean, B, "ymean");
  f32c(w_y, 2 * static_cast<int64_t>(E), "w_y [E, 2]");
  f32c(b_y, E, "b_y");
  AsmArgs a{};
  a.h = reinterpret_cast<const __nv_bfloat16*>(h.data_ptr());
  a.y = y.data_ptr<float>();
  a.ymean = ymean.data_ptr<float>();
  a.use_ta = w_ta.has_value() && w_ta->defined() ? 1 : 0;
  if (a.use_ta) {
    f32c(*w_ta, E, "w_ta");
    f32c(*b_ta, E, "b_ta");
    a.w_ta = w_ta->data_ptr<float>();
    a.b_ta = b_ta->data_ptr<float>();
  }
  a.column_gate = alpha.has_value() && alpha->defined() ? 1 : 0;
  if (a.column_gate) {
    f32c(*alpha, 1, "alpha");
    a.alpha = alpha->data_ptr<float>();
  }
  a.w_y = w_y.data_ptr<float>();
  a.b_y = b_y.data_ptr<float>();
  a.inv_sqrt_e = 1.f / sqrtf(static_cast<float>(E));
  a.ta_scale = static_cast<float>(ta_scale);
  a.B = static_cast<int>(B);
  a.S = static_cast<int>(S);
  a.G = static_cast<int>(G);
  a.E = E;
  a.ep = static_cast<int>(ep);
  a.ylen = static_cast<int>(y.size(1));
  return a;
}

torch::Tensor assemble_fwd(const torch::Tensor& h, const torch::Tensor& y, const torch::Tensor& ymean,
                           const c10::optional<torch::Tensor>& w_ta, const c10::optional<torch::Tensor>& b_ta,
                           const c10::optional<torch::Tensor>& alpha, const torch::Tensor& w_y, const torch::Tensor& b_y,
                           int64_t B, int64_t S, int64_t G, int64_t ep, double ta_scale) {
  AsmArgs a = asm_args(h, y, ymean, w_ta, b_ta, alpha, w_y, b_y, B, S, G, ep, ta_scale);
  const at::cuda::CUDAGuard guard(h.device());
  auto X = torch::empty({B * S * (G + 1), a.E}, h.options());
  if (B * S == 0) return X;
  assemble_fwd_kernel<<<static_cast<unsigned>((B * S + 7) / 8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      a, reinterpret_cast<__nv_bfloat16*>(X.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return X;
}

torch::Tensor assemble_bwd(const torch::Tensor& dX, const torch::Tensor& h, const torch::Tensor& y,
                           const torch::Tensor& ymean, const c10::optional<torch::Tensor>& w_ta,
                           const c10::optional<torch::Tensor>& b_ta, const c10::optional<torch::Tensor>& alpha,
                           const torch::Tensor& w_y, const torch::Tensor& b_y, int64_t B, int64_t S, int64_t G,
                           int64_t ep, double ta_scale, const c10::optional<torch::Tensor>& dw_ta,
                           const c10::optional<torch::Tensor>& db_ta, torch::Tensor& dw_y, torch::Tensor& db_y,
                           const c10::optional<torch::Tensor>& dalpha) {
  AsmArgs a = asm_args(h, y, ymean, w_ta, b_ta, alpha, w_y, b_y, B, S, G, ep, ta_scale);
  TORCH_CHECK(dX.is_cuda() && dX.scalar_type() == at::kBFloat16 && dX.is_contiguous() &&
                  dX.size(0) == B * S * (G + 1) && dX.size(1) == a.E,
              "assemble_bwd: contiguous bf16 dX [R, E]");
  f32c(dw_y, 2 * static_cast<int64_t>(a.E), "dw_y");
  f32c(db_y, a.E, "db_y");
  float *pw = nullptr, *pb = nullptr, *pa = nullptr;
  if (a.use_ta) {
    TORCH_CHECK(dw_ta.has_value() && db_ta.has_value(), "assemble_bwd: target-aware gradient buffers");
    f32c(*dw_ta, a.E, "dw_ta");
    f32c(*db_ta, a.E, "db_ta");
    pw = dw_ta->data_ptr<float>();
    pb = db_ta->data_ptr<float>();
  }
  if (a.column_gate && dalpha.has_value() && dalpha->defined()) {
    f32c(*dalpha, 1, "dalpha");
    pa = dalpha->data_ptr<float>();
  }
  const at::cuda::CUDAGuard guard(h.device());
  auto dh = torch::empty_like(h);
  if (B * S == 0) return dh;
  assemble_bwd_kernel<<<static_cast<unsigned>((B * S + 7) / 8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      a, reinterpret_cast<const __nv_bfloat16*>(dX.data_ptr()), reinterpret_cast<__nv_bfloat16*>(dh.data_ptr()), pw,
      pb, dw_y.data_ptr<float>(), db_y.data_ptr<float>(), pa);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dh;
}

}  // namespace nori
