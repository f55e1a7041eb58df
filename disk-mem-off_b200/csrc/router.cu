// Routing stage of the MoE block (K1/K2): fused RMSNorm + router, top-k, the
// deterministic expert-major permutation, GEMM tile lists, and the dispatch
// gather of normalised f16 rows.
//
// Reference arithmetic (disk-mem-off, offload_runtime/executors):
//   rms_norm      _common.py:73-75       h = w * (x / sqrt(mean(x^2) + eps))
//   router        glm4_moe.py:181-183    logits = h @ Wg^T (+ e_score_correction_bias)
//   scoring/top-k glm4_moe.py:185-200    softmax, top-k by prob, renormalise, * scale
//                 qwen3_next.py:278-293  (no bias, no scale)
//   dispatch      glm4_moe.py:206-215    per expert, tokens ascending
// Everything on the routing path is fp32.  The router uses
// logit = (sum_k (w_k x_k) Wg_k) / rms, the same quantity as h @ Wg^T with the
// per-token 1/rms factored out of the sum.  Ranking uses the biased logit
// (softmax is monotone in it); exact ties go to the lower expert id.
//
// Decode (T <= 256): router -> route_tail (one CTA) -> dispatch.
// Prefill:          router -> topk -> perm_hist -> perm_scan -> perm_scatter -> dispatch.
#include <float.h>

#include <algorithm>

#include "common.cuh"
#include "moe_internal.h"

namespace moe {

// ------------------------------------------------------------------ router
constexpr int kRouterKc = 128;      // K elements per chunk
constexpr int kRouterRows = 32;     // router rows per CTA
constexpr int kRouterPad = 4;       // smem row padding (floats)

MOE_DEV void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}

// sum_{q < n} p[q * stride], added in order q = 0, 1, ...; the loads of a batch
// of 8 are issued before any is added, so a long split count costs a few
// memory latencies rather than one per split.
MOE_DEV float sum_splits(const float* p, size_t stride, int n) {
  float acc = 0.f;
  int q = 0;
  for (; q + 8 <= n; q += 8) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = p[(q + i) * stride];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc += v[i];
  }
  for (; q < n; ++q) acc += p[q * stride];
  return acc;
}

// CTA (rx, s, tz) computes router rows [32 rx, 32 rx + 32) for tokens
// [BT tz, BT tz + BT) over K split s, in chunks of 128 that are requested with
// cp.async all at once (one memory latency per chunk).  It also sums x^2 of its
// tokens over its K range.  With S > 1 splits the partials go to scratch and the
// CTA that finishes last for a (rx, tz) tile adds them in split order
// s = 0..S-1 (deterministic), divides by rms and writes the logits.
template <int BT>
__global__ void __launch_bounds__(256) router_kernel(
    const float* __restrict__ x, const float* __restrict__ wn, const float* __restrict__ wr,
    float* __restrict__ part, float* __restrict__ ss_part, float* __restrict__ logits,
    float* __restrict__ rms_out, int* __restrict__ counters, int T, int H, int R, int S,
    int k_per_split, float eps) {
  pdl_enter();
  constexpr int EPT = (BT == 64) ? 4 : 2;     // router rows per thread
  constexpr int XT = kRouterRows / EPT;       // threads along rows
  constexpr int YT = 256 / XT;                // threads along tokens
  constexpr int TPT = BT / YT;                // tokens per thread
  constexpr int LD = kRouterKc + kRouterPad;  // smem row stride (floats)
  constexpr int TPTOK = 256 / BT;             // threads per token for the x^2 sum
  constexpr int SSV = kRouterKc / 4 / TPTOK;  // float4 per thread per chunk for x^2
  extern __shared__ __align__(16) float rsm[];
  float* xs = rsm;                       // [BT][LD] raw x
  float* ws = xs + BT * LD;              // [32][LD] router rows
  float* wns = ws + kRouterRows * LD;    // [128] norm weight chunk
  __shared__ float s_rms[BT];
  __shared__ int s_last;
  const int rx = blockIdx.x, sp = blockIdx.y, tz = blockIdx.z;
  const int r0 = rx * kRouterRows;
  const int t0 = tz * BT;
  const int kb = sp * k_per_split;
  const int ke = min(H, kb + k_per_split);
  const int tid = threadIdx.x;
  const int ty = tid / XT, tx = tid % XT;
  const int stok = tid / TPTOK, sseg = tid % TPTOK;
  float acc[TPT][EPT] = {};
  float ss = 0.f;
  for (int k0 = kb; k0 < ke; k0 += kRouterKc) {
    const int nv = min(kRouterKc, ke - k0) >> 2;  // float4 per row (H % 16 == 0)
    for (int i = tid; i < BT * (kRouterKc / 4); i += 256) {
      const int row = i / (kRouterKc / 4), v = i % (kRouterKc / 4);
      float* dst = xs + row * LD + v * 4;
      if (t0 + row < T && v < nv) cp_async16(dst, x + static_cast<size_t>(t0 + row) * H + k0 + v * 4);
      else *reinterpret_cast<float4*>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int i = tid; i < kRouterRows * (kRouterKc / 4); i += 256) {
      const int row = i / (kRouterKc / 4), v = i % (kRouterKc / 4);
      float* dst = ws + row * LD + v * 4;
      if (r0 + row < R && v < nv) cp_async16(dst, wr + static_cast<size_t>(r0 + row) * H + k0 + v * 4);
      else *reinterpret_cast<float4*>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (tid < kRouterKc / 4) {
      float* dst = wns + tid * 4;
      if (tid < nv) cp_async16(dst, wn + k0 + tid * 4);
      else *reinterpret_cast<float4*>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    __syncthreads();
#pragma unroll
    for (int v = 0; v < SSV; ++v) {
      const float4 a = *reinterpret_cast<const float4*>(xs + stok * LD + (sseg * SSV + v) * 4);
      ss = fmaf(a.x, a.x, ss);
      ss = fmaf(a.y, a.y, ss);
      ss = fmaf(a.z, a.z, ss);
      ss = fmaf(a.w, a.w, ss);
    }
#pragma unroll 4
    for (int k = 0; k < kRouterKc; k += 4) {
      const float4 g = *reinterpret_cast<const float4*>(wns + k);
      float4 a[TPT], b[EPT];
#pragma unroll
      for (int i = 0; i < TPT; ++i) {
        const float4 xv = *reinterpret_cast<const float4*>(xs + (ty + YT * i) * LD + k);
        a[i] = make_float4(g.x * xv.x, g.y * xv.y, g.z * xv.z, g.w * xv.w);
      }
#pragma unroll
      for (int j = 0; j < EPT; ++j) b[j] = *reinterpret_cast<const float4*>(ws + (tx + XT * j) * LD + k);
#pragma unroll
      for (int i = 0; i < TPT; ++i)
#pragma unroll
        for (int j = 0; j < EPT; ++j) {
          float c = acc[i][j];
          c = fmaf(a[i].x, b[j].x, c);
          c = fmaf(a[i].y, b[j].y, c);
          c = fmaf(a[i].z, b[j].z, c);
          c = fmaf(a[i].w, b[j].w, c);
          acc[i][j] = c;
        }
    }
    __syncthreads();
  }
  // x^2 of token stok over this split: reduce the TPTOK consecutive lanes
#pragma unroll
  for (int o = TPTOK / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);

  if (S == 1) {  // whole K in this CTA: finish directly
    if (sseg == 0) s_rms[stok] = sqrtf(ss / static_cast<float>(H) + eps);
    __syncthreads();
#pragma unroll
    for (int i = 0; i < TPT; ++i) {
      const int tl = ty + YT * i, t = t0 + tl;
      if (t >= T) continue;
#pragma unroll
      for (int j = 0; j < EPT; ++j) {
        const int r = r0 + tx + XT * j;
        if (r < R) logits[static_cast<size_t>(t) * R + r] = acc[i][j] / s_rms[tl];
      }
    }
    if (rx == 0 && sseg == 0 && t0 + stok < T) rms_out[t0 + stok] = s_rms[stok];
    return;
  }

  float* out = part + static_cast<size_t>(sp) * T * R;
#pragma unroll
  for (int i = 0; i < TPT; ++i) {
    const int t = t0 + ty + YT * i;
    if (t >= T) continue;
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
      const int r = r0 + tx + XT * j;
      if (r < R) out[static_cast<size_t>(t) * R + r] = acc[i][j];
    }
  }
  if (sseg == 0 && t0 + stok < T) ss_part[(static_cast<size_t>(rx) * S + sp) * T + t0 + stok] = ss;
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = (atomicAdd(&counters[rx * gridDim.z + tz], 1) == S - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (tid < BT && t0 + tid < T) {
    const float tot = sum_splits(ss_part + static_cast<size_t>(rx) * S * T + t0 + tid,
                                 static_cast<size_t>(T), S);
    s_rms[tid] = sqrtf(tot / static_cast<float>(H) + eps);
    if (rx == 0) rms_out[t0 + tid] = s_rms[tid];
  }
  __syncthreads();
  for (int o = tid; o < BT * kRouterRows; o += 256) {
    const int tl = o / kRouterRows, r = r0 + o % kRouterRows, t = t0 + tl;
    if (t >= T || r >= R) continue;
    const float v = sum_splits(part + static_cast<size_t>(t) * R + r, static_cast<size_t>(T) * R, S);
    logits[static_cast<size_t>(t) * R + r] = v / s_rms[tl];
  }
}

// ------------------------------------------------------------------ top-k
// One warp scores and selects for one token.  Lane l holds experts l, l+32, ...
// Keys rank (desc) with the lower id winning exact ties; weights follow the
// reference formulas in fp32.  Lane r < K writes ids_out[r] / w_out[r].
template <int VPL>
MOE_DEV void warp_topk(const float* __restrict__ lrow, const float* __restrict__ bias, int E,
                       int K, int score_func, int norm, float scale, int lane,
                       int32_t* ids_out, float* w_out, int* err) {
  // every load first (one memory round trip, not one per value), then the scores
  float lv[VPL], bv0[VPL];
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int e = j * 32 + lane;
    lv[j] = e < E ? lrow[e] : 0.f;
    bv0[j] = (bias && e < E) ? bias[e] : 0.f;
  }
  float key[VPL], val[VPL];
  float m = -FLT_MAX;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int e = j * 32 + lane;
    key[j] = -FLT_MAX;
    val[j] = 0.f;
    if (e < E) {
      float l = lv[j];
      if (score_func == MOE_SCORE_SOFTMAX) {
        if (bias) l = l + bv0[j];
        key[j] = l;
        val[j] = l;
        m = fmaxf(m, l);
      } else {
        const float s = sigmoid_f(l);
        val[j] = s;
        key[j] = bias ? s + bv0[j] : s;
      }
    }
  }
  float denom = 1.f;
  if (score_func == MOE_SCORE_SOFTMAX) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      if (j * 32 + lane < E) {
        val[j] = expf(val[j] - m);
        s += val[j];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    denom = s;
  }
  // Each candidate as one 64-bit key: the score's bits in an order-preserving
  // form above the complemented expert id, so one unsigned max picks the largest
  // score and, among equal scores, the lowest id.  Lane r keeps the r-th selection.
  uint64_t pk[VPL];
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int e = j * 32 + lane;
    if (e < E) {
      const uint32_t u = __float_as_uint(key[j]);
      const uint32_t ob = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
      pk[j] = (static_cast<uint64_t>(ob) << 32) | static_cast<uint32_t>(~e);
    } else {
      pk[j] = 0ull;
    }
  }
  int my_id = 0;
  float my_w = 0.f;
  for (int r = 0; r < K; ++r) {
    uint64_t best = 0ull;
#pragma unroll
    for (int j = 0; j < VPL; ++j) best = pk[j] > best ? pk[j] : best;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    int bid = static_cast<int>(~static_cast<uint32_t>(best));
    if (best == 0ull || bid < 0 || bid >= E) {  // K > E cannot happen for a validated plan
      record_error(err, DEV_BAD_ROUTE);
      bid = 0;
    }
    const int slot = bid >> 5;
    float v = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) v = (j == slot) ? val[j] : v;
    const float bv = __shfl_sync(0xffffffffu, v, bid & 31);
    if (lane == r) {
      my_id = bid;
      my_w = (score_func == MOE_SCORE_SOFTMAX) ? bv / denom : bv;
    }
    if ((bid & 31) == lane) {
#pragma unroll
      for (int j = 0; j < VPL; ++j) pk[j] = (j == slot) ? 0ull : pk[j];
    }
  }
  float sum = 0.f;  // rank order, one term at a time
  if (norm)
    for (int r = 0; r < K; ++r) sum += __shfl_sync(0xffffffffu, my_w, r);
  if (lane < K) {
    float wv = my_w;
    if (norm) wv = wv / (sum + 1e-20f);
    ids_out[lane] = my_id;
    w_out[lane] = wv * scale;
  }
}

// Prefill tensor-core router, selection stage.  The tensor-core logits use f16
// operands (~2e-3 absolute error at most for GLM-4.7 shapes, 2.5e-4 typical),
// so they only choose candidates; the decision is made on fp32 logits
// recomputed on the CUDA cores (sum_k (w_k x_k) Wg_k / rms, in a fixed order),
// in three launches:
//   route_cand_kernel   warp per token: adds the logit planes (into plane 0),
//                       takes the C = K + kRefineMargin best tensor-core keys
//                       and names the rows to recompute: the K chosen experts
//                       plus every candidate whose key is within kRefineGap *
//                       max(1, |best key|) of the K-th key (usually none or
//                       one); every expert when even the C-th key is that
//                       close (ties across the whole window).
//   route_exact_kernel  CTA per token, warp per row: fp32 dot products against
//                       the token's normalised row, staged once in shared
//                       memory, with sixteen loads of the router row in flight
//                       per lane; writes the exact logits (plane 0's row when
//                       every expert is recomputed) and the shared-expert gate
//                       logit.
//   route_final_kernel  warp per token: softmax over all experts with the
//                       exact logits substituted, top-k among the recomputed
//                       rows by exact keys and the lower-id tie rule, weights.
// kRefineGap is ~4x the largest f16 logit error seen: an expert outside the
// recomputed set is more than the gap below the K-th key, so the selection,
// order and weights are those of the fp32 router.
constexpr float kRefineGap = 8e-3f;
static_assert(kCandMax <= 64, "route_final_kernel holds two candidate slots per lane");

template <int VPL>
__global__ void __launch_bounds__(256) route_cand_kernel(
    float* __restrict__ logits, int nplanes, const float* __restrict__ bias,
    int32_t* __restrict__ cand, int32_t* __restrict__ nrows, int T, int E, int R, int K,
    int score_func, int* err) {
  pdl_enter();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  const size_t plane = static_cast<size_t>(T) * R;
  float* lrow = logits + static_cast<size_t>(t) * R;
  const int C = min(E, K + kRefineMargin);
  // all plane and bias loads are issued before any is used (the bounds are constants)
  float pl[kRouterMaxSplit][VPL];
  float bs[VPL];
#pragma unroll
  for (int sp = 0; sp < kRouterMaxSplit; ++sp)
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int e = j * 32 + lane;
      pl[sp][j] = (sp < nplanes && e < E) ? lrow[sp * plane + e] : 0.f;
    }
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int e = j * 32 + lane;
    bs[j] = (bias && e < E) ? bias[e] : 0.f;
  }
  // each candidate as one 64-bit key (order-preserving score bits over the
  // complemented id): one unsigned max per round picks the largest key and, among
  // equal keys, the lowest id; a NaN key is reported and never selected
  uint64_t pk[VPL];
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int e = j * 32 + lane;
    pk[j] = 0ull;
    if (e < E) {
      float l = pl[0][j];
#pragma unroll
      for (int sp = 1; sp < kRouterMaxSplit; ++sp)
        if (sp < nplanes) l += pl[sp][j];  // split order
      if (nplanes > 1) lrow[e] = l;  // plane 0 now holds the summed logits
      const float key = (score_func == MOE_SCORE_SOFTMAX) ? (bias ? l + bs[j] : l)
                                                          : (bias ? sigmoid_f(l) + bs[j] : sigmoid_f(l));
      if (key != key) {
        record_error(err, DEV_BAD_ROUTE);
      } else {
        const uint32_t u = __float_as_uint(key);
        const uint32_t ob = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
        pk[j] = (static_cast<uint64_t>(ob) << 32) | static_cast<uint32_t>(~e);
      }
    }
  }
  if (nplanes > 1 && lane == 0 && E < R) {  // the shared-expert gate row
    float l = lrow[E];
    for (int sp = 1; sp < nplanes; ++sp) l += lrow[sp * plane + E];
    lrow[E] = l;
  }
  float thr = 0.f, k_last = 0.f;
  int n = K;
  bool all_rows = false;
  for (int r = 0; r < C; ++r) {
    uint64_t best = 0ull;
#pragma unroll
    for (int j = 0; j < VPL; ++j) best = pk[j] > best ? pk[j] : best;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    int bid = static_cast<int>(~static_cast<uint32_t>(best));
    const uint32_t ob = static_cast<uint32_t>(best >> 32);
    const float bk = __uint_as_float((ob & 0x80000000u) ? (ob & 0x7fffffffu) : ~ob);
    if (best == 0ull || bid < 0 || bid >= E) {  // no selectable key left (NaN keys)
      record_error(err, DEV_BAD_ROUTE);
      bid = 0;
    }
    if (r == 0) thr = kRefineGap * fmaxf(1.f, fabsf(bk));
    if (r == K - 1) k_last = bk;
    if (r >= K) {
      if (k_last - bk < thr) {
        n = r + 1;  // still inside the tie window
        if (r == C - 1 && C < E) all_rows = true;
      } else {
        break;  // keys only fall from here on
      }
    }
    const bool mine = lane == (bid & 31);
    const int slot = bid >> 5;
#pragma unroll
    for (int j = 0; j < VPL; ++j) pk[j] = (mine && j == slot) ? 0ull : pk[j];
    if (lane == 0) cand[static_cast<size_t>(t) * kCandMax + r] = bid;
  }
  if (lane == 0) nrows[t] = all_rows ? -1 : n;
}

// Rows of token t: its n candidates (then the gate row E when the layer has a
// shared-expert gate), or all R router rows when n < 0.
__global__ void __launch_bounds__(256) route_exact_kernel(
    float* __restrict__ logits, const int32_t* __restrict__ cand, const int32_t* __restrict__ nrows,
    const float* __restrict__ x, const float* __restrict__ wn, const float* __restrict__ wr,
    const float* __restrict__ rms, float* __restrict__ exact, int T, int E, int R, int H,
    int has_gate) {
  pdl_enter();
  extern __shared__ float4 s_u[];  // [H / 4]: wn * x of this token
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = nrows[t];
  const bool all_rows = n < 0;
  const int rows = all_rows ? R : n + (has_gate ? 1 : 0);
  const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(t) * H);
  const float4* gr = reinterpret_cast<const float4*>(wn);
  const int nv = H >> 2;
  const float rt = rms[t];
  auto row_of = [&](int r) {
    if (all_rows) return r;
    return r < n ? cand[static_cast<size_t>(t) * kCandMax + r] : E;
  };
  for (int v = threadIdx.x; v < nv; v += blockDim.x) {
    const float4 xv = xr[v], g = __ldg(gr + v);
    s_u[v] = make_float4(g.x * xv.x, g.y * xv.y, g.z * xv.z, g.w * xv.w);
  }
  __syncthreads();
  // a row per warp, sixteen float4 of it in flight per lane; each lane adds its
  // columns k = lane (mod 32) in ascending order, then the warp's shuffle tree
  for (int r = warp; r < rows; r += 8) {
    const float4* w = reinterpret_cast<const float4*>(wr + static_cast<size_t>(row_of(r)) * H);
    float a = 0.f;
    int k = lane;
    for (; k + 32 * 15 < nv; k += 32 * 16) {
      float4 p[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) p[i] = __ldg(w + k + 32 * i);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 u = s_u[k + 32 * i];
        a = fmaf(u.x, p[i].x, a);
        a = fmaf(u.y, p[i].y, a);
        a = fmaf(u.z, p[i].z, a);
        a = fmaf(u.w, p[i].w, a);
      }
    }
    for (; k < nv; k += 32) {
      const float4 u = s_u[k], p = __ldg(w + k);
      a = fmaf(u.x, p.x, a);
      a = fmaf(u.y, p.y, a);
      a = fmaf(u.z, p.z, a);
      a = fmaf(u.w, p.w, a);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (lane == 0) {
      const float v = a / rt;
      if (all_rows) logits[static_cast<size_t>(t) * R + r] = v;  // plane 0's row becomes exact
      else exact[static_cast<size_t>(t) * (kCandMax + 1) + r] = v;
    }
  }
}

template <int VPL>
__global__ void __launch_bounds__(256) route_final_kernel(
    const float* __restrict__ logits, const int32_t* __restrict__ cand,
    const int32_t* __restrict__ nrows, const float* __restrict__ exact,
    const float* __restrict__ bias, int32_t* __restrict__ ids, float* __restrict__ wts,
    float* __restrict__ sgate, int T, int E, int R, int K, int score_func, int norm, float scale,
    int* err) {
  pdl_enter();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  const float* lrow = logits + static_cast<size_t>(t) * R;
  const int n = nrows[t];
  if (n < 0) {  // every expert recomputed: plane 0's row is exact
    warp_topk<VPL>(lrow, bias, E, K, score_func, norm, scale, lane, ids + static_cast<size_t>(t) * K,
                   wts + static_cast<size_t>(t) * K, err);
    if (sgate && lane == 0) sgate[t] = sigmoid_f(lrow[E]);
    return;
  }
  const int32_t* crow = cand + static_cast<size_t>(t) * kCandMax;
  const float* xrow = exact + static_cast<size_t>(t) * (kCandMax + 1);
  // this lane's recomputed candidates (slots lane, lane + 32)
  float cl[2];
  int ce[2];
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int c = lane + 32 * q;
    ce[q] = c < n ? crow[c] : 0x7fffffff;
    cl[q] = c < n ? xrow[c] : 0.f;
  }
  float denom = 1.f, m = -FLT_MAX;
  if (score_func == MOE_SCORE_SOFTMAX) {
    float lv[VPL];
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int e = j * 32 + lane;
      lv[j] = -FLT_MAX;
      if (e < E) lv[j] = lrow[e];
    }
    // substitute the exact logits of the recomputed candidates
    for (int c = 0; c < n; ++c) {
      const int e = __shfl_sync(0xffffffffu, c < 32 ? ce[0] : ce[1], c & 31);
      const float l = __shfl_sync(0xffffffffu, c < 32 ? cl[0] : cl[1], c & 31);
#pragma unroll
      for (int j = 0; j < VPL; ++j)
        if (j == (e >> 5) && lane == (e & 31)) lv[j] = l;
    }
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int e = j * 32 + lane;
      if (e < E) {
        if (bias) lv[j] = lv[j] + bias[e];
        m = fmaxf(m, lv[j]);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float ssum = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j)
      if (j * 32 + lane < E) ssum += expf(lv[j] - m);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ssum += __shfl_xor_sync(0xffffffffu, ssum, o);
    denom = ssum;
  }
  float ck[2], cv[2];
  int rank[2];
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    ck[q] = -FLT_MAX;
    cv[q] = 0.f;
    rank[q] = -1;
    if (ce[q] != 0x7fffffff) {
      const int e = ce[q];
      const float l = cl[q];
      if (score_func == MOE_SCORE_SOFTMAX) {
        ck[q] = bias ? l + bias[e] : l;
        cv[q] = expf(ck[q] - m) / denom;
      } else {
        cv[q] = sigmoid_f(l);
        ck[q] = bias ? cv[q] + bias[e] : cv[q];
      }
    }
  }
  float sum = 0.f;
  for (int r = 0; r < K; ++r) {
    float bk = -FLT_MAX, bv = 0.f;
    int bid = 0x7fffffff;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      if (ce[q] != 0x7fffffff && rank[q] < 0 &&
          (bid == 0x7fffffff || ck[q] > bk || (ck[q] == bk && ce[q] < bid))) {
        bk = ck[q];
        bid = ce[q];
        bv = cv[q];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ok = __shfl_xor_sync(0xffffffffu, bk, o);
      const int oid = __shfl_xor_sync(0xffffffffu, bid, o);
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      if (oid != 0x7fffffff && (bid == 0x7fffffff || ok > bk || (ok == bk && oid < bid))) {
        bk = ok;
        bid = oid;
        bv = ov;
      }
    }
    if (bid == 0x7fffffff) {  // fewer than K recomputed rows cannot happen (n >= K)
      record_error(err, DEV_BAD_ROUTE);
      bid = 0;
    }
#pragma unroll
    for (int q = 0; q < 2; ++q)
      if (ce[q] == bid) rank[q] = r;
    if (norm) sum += bv;  // rank order, like warp_topk
  }
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    if (rank[q] >= 0) {
      float wv = cv[q];
      if (norm) wv = wv / (sum + 1e-20f);
      ids[static_cast<size_t>(t) * K + rank[q]] = ce[q];
      wts[static_cast<size_t>(t) * K + rank[q]] = wv * scale;
    }
  }
  if (sgate && lane == 0) sgate[t] = sigmoid_f(xrow[n]);
}

template <int VPL>
__global__ void __launch_bounds__(256) topk_kernel(const float* __restrict__ logits,
                                                   const float* __restrict__ bias,
                                                   int32_t* __restrict__ ids, float* __restrict__ wts,
                                                   float* __restrict__ sgate, int T, int E, int R,
                                                   int K, int score_func, int norm, float scale,
                                                   int* err) {
  pdl_enter();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  const float* lrow = logits + static_cast<size_t>(t) * R;
  warp_topk<VPL>(lrow, bias, E, K, score_func, norm, scale, lane, ids + static_cast<size_t>(t) * K,
                 wts + static_cast<size_t>(t) * K, err);
  if (sgate && lane == 0) sgate[t] = sigmoid_f(lrow[E]);
}

// ------------------------------------------------------------------ tile lists
// Block-wide exclusive scan of one int per thread (blockDim.x == 1024).
__device__ int block_excl_scan(int v, int* total) {
  __shared__ int wsum[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int s = wsum[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    wsum[lane] = s;
  }
  __syncthreads();
  const int incl = x + (warp > 0 ? wsum[warp - 1] : 0);
  if (total) *total = wsum[31];
  __syncthreads();
  return incl - v;
}

struct TileArgs {
  int E, T, bn, mt1, mt2, mt1s, has_shared, max1, max2;
  int shared_group;                // group id the GEMM treats as the shared expert (n_local)
  int nk1, nk1s, nk2, nk2s;        // k-blocks: gate/up routed / shared, down routed / shared
  int num_sms, max_split_tiles;
  int32_t* pre1;                   // [E + 1] gate/up routed tile prefix
  int32_t* pre2;                   // [E + 1] down routed tile prefix
  int32_t* info;                   // [2][4]: routed tiles, K splits, units per GEMM
  int* kcount1;
  int* kcount2;
  int* err;
};

// K splits for a list of `c` tiles on `g` persistent CTAs (each split keeps at
// least kMinSplitKb k-blocks: shorter splits cost more in partial traffic and
// epilogue hand-offs than the better wave fill gains; measured on the GLM-4.7
// down projection, K = 1536).  A list that fits in one wave even when split 4 ways is
// split as far as K allows (less sequential work per CTA); otherwise the
// smallest s <= 4 that fills the last wave best.  Only small lists are split.
constexpr int kMinSplitKb = 16;

MOE_DEV int choose_ksplit(int c, int g, int max_split_tiles, int nk_min) {
  if (c <= 0 || c >= max_split_tiles || g <= 0) return 1;
  if (c * kMaxKSplit <= g) {
    int sp = kMaxKSplit;
    while (sp > 1 && nk_min / sp < kMinSplitKb) --sp;
    return sp;
  }
  int best = 1;
  float best_eff = 0.f;
  for (int sp = 1; sp <= kMaxKSplit; ++sp) {
    if (nk_min / sp < kMinSplitKb) break;
    const int units = c * sp;
    const float eff = static_cast<float>(units) / static_cast<float>(((units + g - 1) / g) * g);
    if (eff > best_eff + 0.02f) {
      best_eff = eff;
      best = sp;
    }
  }
  return best;
}

// Expert e = threadIdx.x owns `cnt` rows.  Writes both GEMMs' tile maps: the
// routed tile prefix over experts (ceil(cnt / bn) token tiles times the weight
// m-tiles), the unit counts with the shared expert's tiles appended, and the K
// split chosen for each list; zeroes the split arrival counters.  Called by
// every thread of a 1024-thread CTA.
__device__ void build_tile_lists(int cnt, const TileArgs& a) {
  __shared__ int s_c[2], s_split[2];
  const int e = threadIdx.x;
  const int ntn = (e < a.E) ? (cnt + a.bn - 1) / a.bn : 0;
  int tot1 = 0, tot2 = 0;
  const int p1 = block_excl_scan(ntn * a.mt1, &tot1);
  const int p2 = block_excl_scan(ntn * a.mt2, &tot2);
  if (e < a.E) {
    a.pre1[e] = p1;
    a.pre2[e] = p2;
  }
  if (e == 0) {
    const int nts = a.has_shared ? (a.T + a.bn - 1) / a.bn : 0;
    const int c1 = tot1 + a.mt1s * nts, c2 = tot2 + a.mt2 * nts;
    const int s1 = choose_ksplit(c1, a.num_sms, a.max_split_tiles, min(a.nk1, a.has_shared ? a.nk1s : a.nk1));
    const int s2 = choose_ksplit(c2, a.num_sms, a.max_split_tiles, min(a.nk2, a.has_shared ? a.nk2s : a.nk2));
    if (c1 > a.max1 || c2 > a.max2) record_error(a.err, DEV_TILE_OVERFLOW);
    a.pre1[a.E] = tot1;
    a.pre2[a.E] = tot2;
    s_c[0] = min(c1, a.max1);
    s_c[1] = min(c2, a.max2);
    s_split[0] = s1;
    s_split[1] = s2;
    a.info[0] = tot1;
    a.info[1] = s1;
    a.info[2] = s_c[0] * s1;
    a.info[4] = tot2;
    a.info[5] = s2;
    a.info[6] = s_c[1] * s2;
  }
  __syncthreads();
  for (int pass = 0; pass < 2; ++pass) {
    if (s_split[pass] > 1) {
      int* kcount = pass ? a.kcount2 : a.kcount1;
      for (int q = threadIdx.x; q < s_c[pass]; q += blockDim.x) kcount[q] = 0;
    }
  }
}

// ------------------------------------------------------------------ decode tail
// One CTA (1024 threads) for T <= kTailMaxT: top-k of every token (a warp per
// token), per-expert token bitmasks, expert offsets, tile lists and the
// (token, slot) -> row permutation.  The rank of a token inside its expert is
// the popcount of the lower bits of the expert's mask, so the dispatch order
// (tokens ascending) is deterministic without ordering any atomics.
template <int VPL>
__global__ void __launch_bounds__(1024) route_tail_kernel(
    const float* __restrict__ logits, const float* __restrict__ bias, int T, int E, int R, int K,
    int score_func, int norm, float scale, int32_t* __restrict__ ids, float* __restrict__ wts,
    float* __restrict__ sgate, int32_t* __restrict__ offsets, int32_t* __restrict__ perm,
    int32_t* __restrict__ slot_row, TileArgs ta) {
  pdl_enter();
  extern __shared__ int tsm[];
  const int words = (T + 31) >> 5;
  int* s_ids = tsm;                                              // [T*K]
  uint32_t* bm = reinterpret_cast<uint32_t*>(s_ids + T * K);     // [E][words]
  int* s_off = reinterpret_cast<int*>(bm + E * words);           // [E]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < E * words; i += blockDim.x) bm[i] = 0u;
  for (int t = warp; t < T; t += 32) {
    const float* lrow = logits + static_cast<size_t>(t) * R;
    warp_topk<VPL>(lrow, bias, E, K, score_func, norm, scale, lane, s_ids + t * K,
                   wts + static_cast<size_t>(t) * K, ta.err);
    if (sgate && lane == 0) sgate[t] = sigmoid_f(lrow[E]);
  }
  __syncthreads();
  for (int q = threadIdx.x; q < T * K; q += blockDim.x) {
    const int e = s_ids[q];
    ids[q] = e;
    const int t = q / K;
    atomicOr(&bm[e * words + (t >> 5)], 1u << (t & 31));
  }
  __syncthreads();
  int cnt = 0;
  if (threadIdx.x < E)
    for (int w = 0; w < words; ++w) cnt += __popc(bm[threadIdx.x * words + w]);
  int all = 0;
  const int off = block_excl_scan(threadIdx.x < E ? cnt : 0, &all);
  if (threadIdx.x < E) {
    offsets[threadIdx.x] = off;
    s_off[threadIdx.x] = off;
  }
  if (threadIdx.x == 0) offsets[E] = all;
  build_tile_lists(cnt, ta);
  __syncthreads();
  for (int q = threadIdx.x; q < T * K; q += blockDim.x) {
    const int e = s_ids[q];
    const int t = q / K;
    const uint32_t* row = bm + e * words;
    int rank = __popc(row[t >> 5] & ((1u << (t & 31)) - 1u));
    for (int w = 0; w < (t >> 5); ++w) rank += __popc(row[w]);
    const int r = s_off[e] + rank;
    perm[r] = q;
    slot_row[q] = r;
  }
}

// ------------------------------------------------------------------ small decode batches
// Batches of up to kSmallT tokens route in ONE launch: the router GEMV, top-k,
// permutation and tile maps, where the launches above take two (a split-K router
// with a last-CTA reduction, then the one-CTA tail), each a few microseconds of
// launch, wait and reduction latency that a one-token step cannot hide.
//   every CTA: x_t * norm_w for the batch into shared memory (and sum x^2 for the
//              RMS), then each warp one router row: logit = sum_k (w_k x_k) r_k / rms
//   the CTA that finishes last (a counter): top-k of every token (a warp per
//              token), expert bitmasks, offsets, the (token, slot) permutation and
//              both GEMMs' tile maps, as route_tail_kernel does.
#ifndef MOE_SMALL_ROUTE_MAX_T
#define MOE_SMALL_ROUTE_MAX_T 8
#endif
constexpr int kSmallT = 8;
constexpr int kSmallRowsPerCta = 8;  // one router row per warp

// Exclusive scan of one int per thread for any block size that is a multiple of
// 32 (up to 1024); every thread gets the block total in *total.
__device__ int block_excl_scan_any(int v, int* total) {
  __shared__ int wsum[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nw ? wsum[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    wsum[lane] = w;
  }
  __syncthreads();
  const int incl = x + (warp > 0 ? wsum[warp - 1] : 0);
  *total = wsum[31];
  __syncthreads();
  return incl - v;
}

// In-place exclusive scan of a[0, n) in shared memory by the whole block (each
// thread a contiguous run); returns the total.
__device__ int block_scan_smem(int* a, int n) {
  const int per = (n + blockDim.x - 1) / blockDim.x;
  const int beg = min(n, threadIdx.x * per), end = min(n, beg + per);
  int sum = 0;
  for (int i = beg; i < end; ++i) sum += a[i];
  int total = 0;
  int run = block_excl_scan_any(sum, &total);
  for (int i = beg; i < end; ++i) {
    const int v = a[i];
    a[i] = run;
    run += v;
  }
  __syncthreads();
  return total;
}

// build_tile_lists for any block size, from per-expert row counts in shared memory
// (s_cnt[E]); s_a / s_b are E-entry shared scratch arrays.
__device__ void build_tile_lists_smem(const int* s_cnt, int* s_a, int* s_b, const TileArgs& a) {
  __shared__ int s_c[2], s_split[2];
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) {
    const int ntn = (s_cnt[e] + a.bn - 1) / a.bn;
    s_a[e] = ntn * a.mt1;
    s_b[e] = ntn * a.mt2;
  }
  __syncthreads();
  const int tot1 = block_scan_smem(s_a, a.E);
  const int tot2 = block_scan_smem(s_b, a.E);
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) {
    a.pre1[e] = s_a[e];
    a.pre2[e] = s_b[e];
  }
  if (threadIdx.x == 0) {
    const int nts = a.has_shared ? (a.T + a.bn - 1) / a.bn : 0;
    const int c1 = tot1 + a.mt1s * nts, c2 = tot2 + a.mt2 * nts;
    const int s1 = choose_ksplit(c1, a.num_sms, a.max_split_tiles, min(a.nk1, a.has_shared ? a.nk1s : a.nk1));
    const int s2 = choose_ksplit(c2, a.num_sms, a.max_split_tiles, min(a.nk2, a.has_shared ? a.nk2s : a.nk2));
    if (c1 > a.max1 || c2 > a.max2) record_error(a.err, DEV_TILE_OVERFLOW);
    a.pre1[a.E] = tot1;
    a.pre2[a.E] = tot2;
    s_c[0] = min(c1, a.max1);
    s_c[1] = min(c2, a.max2);
    s_split[0] = s1;
    s_split[1] = s2;
    a.info[0] = tot1;
    a.info[1] = s1;
    a.info[2] = s_c[0] * s1;
    a.info[4] = tot2;
    a.info[5] = s2;
    a.info[6] = s_c[1] * s2;
  }
  __syncthreads();
  for (int pass = 0; pass < 2; ++pass) {
    if (s_split[pass] > 1) {
      int* kcount = pass ? a.kcount2 : a.kcount1;
      for (int q = threadIdx.x; q < s_c[pass]; q += blockDim.x) kcount[q] = 0;
    }
  }
}

template <int VPL>
__global__ void __launch_bounds__(256) route_small_kernel(
    const float* __restrict__ x, const float* __restrict__ wn, const float* __restrict__ wr,
    const float* __restrict__ bias, int T, int H, int E, int R, int K, int score_func, int norm,
    float scale, float eps, float* __restrict__ logits, float* __restrict__ rms_out,
    int* __restrict__ counter, int32_t* __restrict__ ids, float* __restrict__ wts,
    float* __restrict__ sgate, int32_t* __restrict__ offsets, int32_t* __restrict__ perm,
    int32_t* __restrict__ slot_row, TileArgs ta) {
  pdl_enter();
  extern __shared__ __align__(16) float xs[];  // [T][H]: x * norm weight
  __shared__ float s_rms[kSmallT];
  __shared__ int s_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nv = H >> 2;  // float4 per row
  // the batch's x rows into shared memory, every copy in flight at once
  for (int i = threadIdx.x; i < T * nv; i += blockDim.x) {
    const int t = i / nv, v = i - t * nv;
    cp_async16(xs + static_cast<size_t>(t) * H + 4 * v, x + static_cast<size_t>(t) * H + 4 * v);
  }
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  // sum of x^2 per token and x * norm weight in place; each thread the same
  // float4 columns of every token, so its norm weights are loaded once
  float ss[kSmallT];
#pragma unroll
  for (int t = 0; t < kSmallT; ++t) ss[t] = 0.f;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    const float4 g = reinterpret_cast<const float4*>(wn)[i];
#pragma unroll
    for (int t = 0; t < kSmallT; ++t) {
      if (t < T) {
        float4* p = reinterpret_cast<float4*>(xs + static_cast<size_t>(t) * H) + i;
        const float4 v = *p;
        float q = ss[t];
        q = fmaf(v.x, v.x, q);
        q = fmaf(v.y, v.y, q);
        q = fmaf(v.z, v.z, q);
        q = fmaf(v.w, v.w, q);
        ss[t] = q;
        *p = make_float4(g.x * v.x, g.y * v.y, g.z * v.z, g.w * v.w);
      }
    }
  }
  __shared__ float s_red[8][kSmallT];
#pragma unroll
  for (int t = 0; t < kSmallT; ++t) {
    float q = ss[t];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    if (lane == 0) s_red[warp][t] = q;
  }
  __syncthreads();
  if (threadIdx.x < T) {  // warp partials added in warp order
    float tot = 0.f;
    for (int w = 0; w < 8; ++w) tot += s_red[w][threadIdx.x];
    s_rms[threadIdx.x] = sqrtf(tot / static_cast<float>(H) + eps);
  }
  __syncthreads();
  // one router row per warp: T dot products over H, eight row loads in flight per lane
  const int r = blockIdx.x * kSmallRowsPerCta + warp;
  if (r < R) {
    float acc[kSmallT];
#pragma unroll
    for (int t = 0; t < kSmallT; ++t) acc[t] = 0.f;
    const float4* wrow = reinterpret_cast<const float4*>(wr + static_cast<size_t>(r) * H);
    constexpr int U = 8;
    for (int base = lane; base < nv; base += 32 * U) {
      float4 w[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = base + 32 * u;
        w[u] = i < nv ? __ldcs(wrow + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = base + 32 * u;
        if (i >= nv) break;
#pragma unroll
        for (int t = 0; t < kSmallT; ++t) {
          if (t < T) {
            const float4 a = reinterpret_cast<const float4*>(xs + static_cast<size_t>(t) * H)[i];
            float c = acc[t];
            c = fmaf(a.x, w[u].x, c);
            c = fmaf(a.y, w[u].y, c);
            c = fmaf(a.z, w[u].z, c);
            c = fmaf(a.w, w[u].w, c);
            acc[t] = c;
          }
        }
      }
    }
#pragma unroll
    for (int t = 0; t < kSmallT; ++t) {
      if (t < T) {
        float v = acc[t];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) logits[static_cast<size_t>(t) * R + r] = v / s_rms[t];
      }
    }
  }
  // the CTA that finishes last selects, permutes and builds the tile maps
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(counter, 1) == static_cast<int>(gridDim.x) - 1) ? 1 : 0;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  int* s_ids = reinterpret_cast<int*>(xs);  // x is no longer needed: reuse the space
  uint32_t* s_bm = reinterpret_cast<uint32_t*>(s_ids + kSmallT * kMaxTopK);  // [E] token masks
  int* s_cnt = reinterpret_cast<int*>(s_bm + E);
  int* s_a = s_cnt + E;
  int* s_b = s_a + E;
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_bm[e] = 0u;
  if (threadIdx.x < T) rms_out[threadIdx.x] = s_rms[threadIdx.x];
  __syncthreads();
  if (warp < T) {
    const float* lrow = logits + static_cast<size_t>(warp) * R;
    warp_topk<VPL>(lrow, bias, E, K, score_func, norm, scale, lane, s_ids + warp * K,
                   wts + static_cast<size_t>(warp) * K, ta.err);
    if (sgate && lane == 0) sgate[warp] = sigmoid_f(__ldcg(lrow + E));
  }
  __syncthreads();
  for (int q = threadIdx.x; q < T * K; q += blockDim.x) {
    const int e = s_ids[q];
    ids[q] = e;
    atomicOr(&s_bm[e], 1u << (q / K));
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_cnt[e] = __popc(s_bm[e]);
  __syncthreads();
  // offsets: scan of the counts (s_a holds them while the tile maps use s_cnt)
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_a[e] = s_cnt[e];
  __syncthreads();
  const int all = block_scan_smem(s_a, E);
  for (int e = threadIdx.x; e < E; e += blockDim.x) offsets[e] = s_a[e];
  if (threadIdx.x == 0) offsets[E] = all;
  for (int q = threadIdx.x; q < T * K; q += blockDim.x) {
    const int e = s_ids[q], t = q / K;
    const int rr = s_a[e] + __popc(s_bm[e] & ((1u << t) - 1u));
    perm[rr] = q;
    slot_row[q] = rr;
  }
  __syncthreads();
  build_tile_lists_smem(s_cnt, s_a, s_b, ta);
  if (threadIdx.x == 0) *counter = 0;  // ready for the next call
}

// ------------------------------------------------------------------ prefill permutation
// Per chunk of 1024 tokens: a bitmask per expert, written to global with its
// popcount histogram; a single-CTA scan; then one thread per (token, slot).
// Slot q = t * K + k (token t, slot k) has key ids[t * key_ld + k] - key_base.
// allow_pad 1: a negative key marks an unused row (fixed-capacity exchange) and
// is skipped; 2: every key outside [0, E) is skipped (the token-replicated
// exchange, where other ranks own those experts); 0: such a key is an error.
__global__ void __launch_bounds__(1024) perm_hist_kernel(const int32_t* __restrict__ ids, int T,
                                                         int K, int E, int key_ld, int key_base,
                                                         int allow_pad, uint32_t* __restrict__ bmg,
                                                         int32_t* __restrict__ hist, int* err) {
  pdl_enter();
  extern __shared__ uint32_t bm[];  // [E][32]
  const int c = blockIdx.x;
  const int tbeg = c * kPermChunk;
  const int tcnt = min(kPermChunk, T - tbeg);
  for (int i = threadIdx.x; i < E * 32; i += blockDim.x) bm[i] = 0u;
  __syncthreads();
  for (int q = threadIdx.x; q < tcnt * K; q += blockDim.x) {
    const int tl = q / K;
    const int raw = ids[static_cast<size_t>(tbeg + tl) * key_ld + (q - tl * K)];
    const int e = raw - key_base;
    if (e < 0 || e >= E) {
      if (!(allow_pad == 2 || (allow_pad == 1 && raw < 0))) record_error(err, DEV_BAD_ROUTE);
      continue;
    }
    atomicOr(&bm[e * 32 + (tl >> 5)], 1u << (tl & 31));
  }
  __syncthreads();
  uint32_t* out = bmg + static_cast<size_t>(c) * E * 32;
  for (int i = threadIdx.x; i < E * 32; i += blockDim.x) out[i] = bm[i];
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int cnt = 0;
#pragma unroll 8
    for (int w = 0; w < 32; ++w) cnt += __popc(bm[e * 32 + w]);
    hist[static_cast<size_t>(c) * E + e] = cnt;
  }
}

__global__ void __launch_bounds__(1024) perm_scan_kernel(const int32_t* __restrict__ hist,
                                                         int nchunks, int32_t* __restrict__ base,
                                                         int32_t* __restrict__ offsets,
                                                         TileArgs ta) {
  pdl_enter();
  const int e = threadIdx.x, E = ta.E;
  int tot = 0;
  if (e < E) {
    for (int c = 0; c < nchunks; ++c) {
      base[static_cast<size_t>(c) * E + e] = tot;
      tot += hist[static_cast<size_t>(c) * E + e];
    }
  }
  int all = 0;
  const int off = block_excl_scan(e < E ? tot : 0, &all);
  if (e < E) {
    offsets[e] = off;
    for (int c = 0; c < nchunks; ++c) base[static_cast<size_t>(c) * E + e] += off;
  }
  if (e == 0) offsets[E] = all;
  build_tile_lists(tot, ta);
}

__global__ void __launch_bounds__(256) perm_scatter_kernel(const int32_t* __restrict__ ids,
                                                           const uint32_t* __restrict__ bmg,
                                                           const int32_t* __restrict__ base,
                                                           int T, int K, int E, int key_ld,
                                                           int key_base,
                                                           int32_t* __restrict__ perm,
                                                           int32_t* __restrict__ slot_row) {
  pdl_enter();
  for (int q = blockIdx.x * blockDim.x + threadIdx.x; q < T * K; q += gridDim.x * blockDim.x) {
    const int t = q / K;
    const int e = ids[static_cast<size_t>(t) * key_ld + (q - t * K)] - key_base;
    if (e < 0 || e >= E) continue;  // reported by perm_hist_kernel
    const int c = t / kPermChunk, tl = t % kPermChunk;
    const uint32_t* row = bmg + (static_cast<size_t>(c) * E + e) * 32;
    int rank = __popc(row[tl >> 5] & ((1u << (tl & 31)) - 1u));
    for (int w = 0; w < (tl >> 5); ++w) rank += __popc(row[w]);
    const int r = base[static_cast<size_t>(c) * E + e] + rank;
    perm[r] = q;
    slot_row[q] = r;
  }
}

// dst[r] = src[perm[r] / div] for f16 rows of H elements, source rows src_ld
// elements apart (one CTA per row); rows from *nvalid on are left alone when
// nvalid is given (only that many perm entries exist).
__global__ void __launch_bounds__(256) gather_rows_kernel(const __half* __restrict__ src,
                                                          const int32_t* __restrict__ perm, int n,
                                                          int H, int src_ld, int div,
                                                          const int32_t* __restrict__ nvalid,
                                                          __half* __restrict__ dst) {
  pdl_enter();
  if (nvalid) n = min(n, *nvalid);
  for (int r = blockIdx.x; r < n; r += gridDim.x) {
    const uint4* in = reinterpret_cast<const uint4*>(src + static_cast<size_t>(perm[r] / div) * src_ld);
    uint4* out = reinterpret_cast<uint4*>(dst + static_cast<size_t>(r) * H);
    for (int v = threadIdx.x; v < (H >> 3); v += blockDim.x) out[v] = in[v];
  }
}

// ------------------------------------------------------------------ prefill router operands
// Prefill routing prologue, one CTA per token: rms = sqrt(mean(x^2) + eps) and
// h16 = f16(w * (x / rms)), the B operand of the router GEMM and the rows that
// dispatch gathers for the experts.
__global__ void __launch_bounds__(256) router_prep_kernel(const float* __restrict__ x,
                                                          const float* __restrict__ wn, int H,
                                                          float eps, float* __restrict__ rms_out,
                                                          __half* __restrict__ h16, int* err) {
  pdl_enter();
  const int t = blockIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(t) * H);
  const float4* wr = reinterpret_cast<const float4*>(wn);
  const int nv = H >> 2;
  float ss = 0.f;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    const float4 v = xr[i];
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
  }
  __shared__ float red[8];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) tot += red[w];
  const float rms = sqrtf(tot / static_cast<float>(H) + eps);
  if (threadIdx.x == 0) rms_out[t] = rms;
  const float inv = 1.0f / rms;
  __half* hrow = h16 + static_cast<size_t>(t) * H;
  bool bad = false;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    const float4 v = xr[i], g = wr[i];
    __half2 hh[2];
    hh[0] = __floats2half2_rn(g.x * (v.x * inv), g.y * (v.y * inv));
    hh[1] = __floats2half2_rn(g.z * (v.z * inv), g.w * (v.w * inv));
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float2 f = __half22float2(hh[j]);
      bad |= !isfinite(f.x) || !isfinite(f.y);
    }
    reinterpret_cast<uint2*>(hrow)[i] = *reinterpret_cast<uint2*>(hh);
  }
  if (bad) record_error(err, DEV_RANGE);
}

// Bind time: rw16[r] = f16(router row * 2^10); err is set when a weight overflows.
__global__ void __launch_bounds__(256) scale_router_kernel(const float* __restrict__ w,
                                                           __half* __restrict__ rw16, int H,
                                                           int* err) {
  const int r = blockIdx.x;
  const float* row = w + static_cast<size_t>(r) * H;
  __half* out = rw16 + static_cast<size_t>(r) * H;
  bool bad = false;
  for (int k = threadIdx.x; k < H; k += blockDim.x) {
    const __half v = __float2half_rn(row[k] * kRouterWeightScale);
    bad |= !isfinite(__half2float(v));
    out[k] = v;
  }
  if (bad) atomicExch(err, 1);
}

// Dense MLP prologue: rms and the normalised f16 rows (h16) of T tokens.
cudaError_t launch_row_prep(const Plan& p, const WsLayout& L, char* ws, const float* x, int T,
                            cudaStream_t s) {
  MOE_PDL(router_prep_kernel, dim3(T), dim3(256), 0, s, x, p.w.norm_w, p.H, p.cfg.rms_norm_eps,
          reinterpret_cast<float*>(ws + L.rms), reinterpret_cast<__half*>(ws + L.h16), p.d_err);
  return cudaSuccess;
}

cudaError_t launch_norm_rows(const float* x, const float* w, int H, float eps, int T, float* rms,
                             __half* h16, int* err, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  MOE_PDL(router_prep_kernel, dim3(T), dim3(256), 0, s, x, w, H, eps, rms, h16, err);
  return cudaSuccess;
}

cudaError_t launch_scale_router_weights(const float* w, __half* rw16, int rows, int H, int* err,
                                        cudaStream_t s) {
  scale_router_kernel<<<rows, 256, 0, s>>>(w, rw16, H, err);
  return cudaGetLastError();
}

// Prefill batches (the decode tail is not used) route with the tensor-core
// router when the bound router weights fit the scaled f16 split.
bool route_uses_tc_router(const Plan& p, int T) { return p.router_tc && !route_uses_tail(p, T); }

// ------------------------------------------------------------------ dispatch
// dst = f16(w * (x_row / rms)) over H elements, spread over the CTA's threads, 8
// elements per thread per step (the same roundings wherever a row is built).
MOE_DEV void norm_row_f16(const float* __restrict__ x_row, const float* __restrict__ wn, float rms,
                          int H, __half* __restrict__ dst) {
  const float inv = 1.0f / rms;
  const float4* xr = reinterpret_cast<const float4*>(x_row);
  const float4* wr = reinterpret_cast<const float4*>(wn);
  for (int v = threadIdx.x; v < (H >> 3); v += blockDim.x) {
    const float4 a0 = xr[2 * v], a1 = xr[2 * v + 1];
    const float4 g0 = wr[2 * v], g1 = wr[2 * v + 1];
    __half2 o[4];
    o[0] = __floats2half2_rn(g0.x * (a0.x * inv), g0.y * (a0.y * inv));
    o[1] = __floats2half2_rn(g0.z * (a0.z * inv), g0.w * (a0.w * inv));
    o[2] = __floats2half2_rn(g1.x * (a1.x * inv), g1.y * (a1.y * inv));
    o[3] = __floats2half2_rn(g1.z * (a1.z * inv), g1.w * (a1.w * inv));
    reinterpret_cast<uint4*>(dst)[v] = *reinterpret_cast<uint4*>(o);
  }
}

// Rows [0, T*K): xg[r] = f16(w * (x[token(r)] / rms)); rows [T*K, T*K+T): h16[t]
// for the shared expert.  One CTA per row (decode batches have few rows, so
// the row itself is spread over 256 threads).
__global__ void __launch_bounds__(256) dispatch_kernel(const float* __restrict__ x,
                                                       const float* __restrict__ wn,
                                                       const float* __restrict__ rms,
                                                       const int32_t* __restrict__ perm, int T,
                                                       int K, int H, int with_shared,
                                                       __half* __restrict__ xg,
                                                       __half* __restrict__ h16) {
  pdl_enter();
  const int rows = T * K + (with_shared ? T : 0);
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    int t;
    __half* dst;
    if (r < T * K) {
      t = perm[r] / K;
      dst = xg + static_cast<size_t>(r) * H;
    } else {
      t = r - T * K;
      dst = h16 + static_cast<size_t>(t) * H;
    }
    norm_row_f16(x + static_cast<size_t>(t) * H, wn, rms[t], H, dst);
  }
}

// Fixed-capacity send buffer of the expert-parallel exchange: destination rank d
// owns rows [d*cap, (d+1)*cap), each H f16 values and a 16-byte tail whose first
// int32 is the expert id local to d, or -1 for an unused row.  The j-th routed row
// for d (expert-major order, as dispatch_kernel would write it) lands at d*cap + j
// and slot_row records that position for combine.  Rows from world*cap on build
// h16 (shared expert) when with_shared.  Source: x normalised here, or the f16
// rows h16src (prefill routing already built them).
__global__ void __launch_bounds__(256) ep_pack_kernel(
    const float* __restrict__ x, const float* __restrict__ wn, const float* __restrict__ rms,
    const __half* __restrict__ h16src, const int32_t* __restrict__ perm,
    const int32_t* __restrict__ ids, const int32_t* __restrict__ offsets, int T, int K, int H,
    int e_loc, int world, int cap, int with_shared, __half* __restrict__ send,
    int32_t* __restrict__ slot_row, __half* __restrict__ h16, int* err) {
  pdl_enter();
  const size_t ld = static_cast<size_t>(H) + 8;
  const int padded_rows = world * cap;
  const int rows = padded_rows + (with_shared ? T : 0);
  for (int pr = blockIdx.x; pr < rows; pr += gridDim.x) {
    if (pr >= padded_rows) {
      const int t = pr - padded_rows;
      norm_row_f16(x + static_cast<size_t>(t) * H, wn, rms[t], H, h16 + static_cast<size_t>(t) * H);
      continue;
    }
    const int d = pr / cap, j = pr - d * cap;
    const int beg = T > 0 ? offsets[d * e_loc] : 0;
    const int cnt = T > 0 ? offsets[(d + 1) * e_loc] - beg : 0;  // <= cap (host check)
    if (j == 0 && cnt > cap && threadIdx.x == 0) record_error(err, DEV_BAD_TILE);
    __half* row = send + static_cast<size_t>(pr) * ld;
    if (j >= cnt) {
      if (threadIdx.x == 0) *reinterpret_cast<int4*>(row + H) = make_int4(-1, 0, 0, 0);
      continue;
    }
    const int q = perm[beg + j];
    const int t = q / K;
    if (threadIdx.x == 0) {
      *reinterpret_cast<int4*>(row + H) = make_int4(ids[q] - d * e_loc, 0, 0, 0);
      slot_row[q] = pr;
    }
    if (h16src) {
      const uint4* in = reinterpret_cast<const uint4*>(h16src + static_cast<size_t>(t) * H);
      uint4* out = reinterpret_cast<uint4*>(row);
      for (int v = threadIdx.x; v < (H >> 3); v += blockDim.x) out[v] = in[v];
    } else {
      norm_row_f16(x + static_cast<size_t>(t) * H, wn, rms[t], H, row);
    }
  }
}

// Token records of the token-replicated exchange, one CTA per record: H
// normalised f16 values, then the token's K global expert ids (int32) and K
// routing weights (fp32), zero-padded to 16 bytes.  Records T..cap-1 carry id -1
// in every slot (no rank serves them).  With with_shared, h16 (shared expert)
// as well.  Source: x normalised here, or the f16 rows h16src (prefill routing
// already built them).
__global__ void __launch_bounds__(256) ep_token_pack_kernel(
    const float* __restrict__ x, const float* __restrict__ wn, const float* __restrict__ rms,
    const __half* __restrict__ h16src, const int32_t* __restrict__ ids,
    const float* __restrict__ wts, int T, int K, int H, int ld, int cap, int with_shared,
    __half* __restrict__ send, __half* __restrict__ h16) {
  pdl_enter();
  const int tail_words = (ld - H) / 2;  // int32 words after the values
  for (int t = blockIdx.x; t < cap; t += gridDim.x) {
    __half* row = send + static_cast<size_t>(t) * ld;
    int32_t* tail = reinterpret_cast<int32_t*>(row + H);
    for (int i = threadIdx.x; i < tail_words; i += blockDim.x) {
      int32_t v = 0;
      if (i < K) {
        v = t < T ? ids[static_cast<size_t>(t) * K + i] : -1;
      } else if (i < 2 * K && t < T) {
        v = __float_as_int(wts[static_cast<size_t>(t) * K + (i - K)]);
      }
      tail[i] = v;
    }
    if (t >= T) continue;
    if (h16src) {
      const uint4* in = reinterpret_cast<const uint4*>(h16src + static_cast<size_t>(t) * H);
      uint4* out = reinterpret_cast<uint4*>(row);
      for (int v = threadIdx.x; v < (H >> 3); v += blockDim.x) out[v] = in[v];
    } else {
      norm_row_f16(x + static_cast<size_t>(t) * H, wn, rms[t], H, row);
      if (with_shared) norm_row_f16(x + static_cast<size_t>(t) * H, wn, rms[t], H,
                                    h16 + static_cast<size_t>(t) * H);
    }
  }
}

// ------------------------------------------------------------------ launchers
static cudaError_t set_smem_attr(const void* fn, size_t bytes, bool* done) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && done[dev]) return cudaSuccess;
  cudaError_t a = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(bytes));
  if (a == cudaSuccess && dev >= 0 && dev < 64) done[dev] = true;
  return a;
}

// Decode batches use 16-token tiles (more CTAs, shorter last-CTA reductions);
// prefill uses 64-token tiles (4 x 4 outputs per thread).
static int router_bt(int T) { return T <= 64 ? 16 : 64; }

RouterGeom router_geometry(const Plan& p, int T) {
  RouterGeom g;
  const int nchunks = (p.H + kRouterKc - 1) / kRouterKc;
  const int bt = router_bt(T);
  g.rx = (p.router_rows + kRouterRows - 1) / kRouterRows;
  g.tz = (T + bt - 1) / bt;
  // enough CTAs to cover the SMs about twice, never more splits than K chunks
  int s = (2 * p.num_sms + g.rx * g.tz - 1) / (g.rx * g.tz);
  if (s > nchunks) s = nchunks;
  if (s < 1) s = 1;
  const int per = (nchunks + s - 1) / s;
  g.splits = (nchunks + per - 1) / per;  // drop splits that would have no K range
  g.k_per_split = per * kRouterKc;
  return g;
}

template <int BT>
static cudaError_t run_router(const Plan& p, const WsLayout& L, char* ws, const float* x, int T,
                              cudaStream_t s) {
  constexpr size_t smem =
      (static_cast<size_t>(BT + kRouterRows) * (kRouterKc + kRouterPad) + kRouterKc) * sizeof(float);
  static bool done[64] = {};
  cudaError_t a = set_smem_attr(reinterpret_cast<const void*>(router_kernel<BT>), smem, done);
  if (a != cudaSuccess) return a;
  const RouterGeom g = router_geometry(p, T);
  int* counters = reinterpret_cast<int*>(ws + L.counters);
  if (g.splits > 1) {  // the last-CTA counters must start at zero on every call
    a = cudaMemsetAsync(counters, 0, static_cast<size_t>(g.rx) * g.tz * sizeof(int), s);
    if (a != cudaSuccess) return a;
  }
  dim3 grid(g.rx, g.splits, g.tz);
  MOE_PDL(router_kernel<BT>, dim3(grid), dim3(256), smem, s, 
      x, p.w.norm_w, p.w.router_w, reinterpret_cast<float*>(ws + L.part),
      reinterpret_cast<float*>(ws + L.ss_part), reinterpret_cast<float*>(ws + L.logits),
      reinterpret_cast<float*>(ws + L.rms), counters, T, p.H, p.router_rows, g.splits,
      g.k_per_split, p.cfg.rms_norm_eps);
  return cudaGetLastError();
}

static TileArgs tile_args(const Plan& p, const WsLayout& L, char* ws, int T, int groups,
                          bool shared) {
  TileArgs ta;
  ta.E = groups;
  ta.T = T;
  ta.bn = L.bn;
  ta.mt1 = (2 * p.I + kBM - 1) / kBM;
  ta.mt2 = (p.H + kBM - 1) / kBM;
  ta.mt1s = (shared && p.SI > 0) ? (2 * p.SI + kBM - 1) / kBM : 0;
  ta.has_shared = shared && p.SI > 0;
  ta.shared_group = p.n_local;
  ta.max1 = L.max_tiles1;
  ta.max2 = L.max_tiles2;
  ta.nk1 = (p.H + kBK - 1) / kBK;
  ta.nk1s = ta.nk1;
  ta.nk2 = (p.I + kBK - 1) / kBK;
  ta.nk2s = p.SI > 0 ? (p.SI + kBK - 1) / kBK : ta.nk2;
  ta.num_sms = p.num_sms;
  ta.max_split_tiles = L.max_split_tiles;
  ta.pre1 = reinterpret_cast<int32_t*>(ws + L.tile_pre);
  ta.pre2 = ta.pre1 + (groups + 1);
  ta.info = reinterpret_cast<int32_t*>(ws + L.tile_info);
  ta.kcount1 = reinterpret_cast<int*>(ws + L.kcount1);
  ta.kcount2 = reinterpret_cast<int*>(ws + L.kcount2);
  ta.err = p.d_err;
  return ta;
}

bool route_uses_tail(const Plan& p, int T) { return T <= kTailMaxT && T * p.K <= 8192; }

// The one-launch router: small batches whose x rows fit shared memory (8 tokens of
// GLM-4.7's 5120 features = 160 KiB) and whose slot bookkeeping fits the space it
// reuses afterwards.
bool route_uses_small(const Plan& p, int T) {
  if (T > kSmallT || T > MOE_SMALL_ROUTE_MAX_T || p.E == 0) return false;
  const size_t xs = static_cast<size_t>(T) * p.H * 4;
  const size_t tail = (static_cast<size_t>(kSmallT) * kMaxTopK + 4 * static_cast<size_t>(p.E)) * 4;
  return std::max(xs, tail) <= 200 * 1024;
}

static cudaError_t launch_route_small(const Plan& p, const WsLayout& L, char* ws, const float* x,
                                      int T, cudaStream_t s) {
  const int E = p.E, K = p.K, R = p.router_rows;
  int* counter = reinterpret_cast<int*>(ws + L.counters);
  cudaError_t st = cudaMemsetAsync(counter, 0, sizeof(int), s);
  if (st != cudaSuccess) return st;
  const size_t smem = std::max(static_cast<size_t>(T) * p.H * 4,
                               (static_cast<size_t>(kSmallT) * kMaxTopK + 4 * static_cast<size_t>(E)) * 4);
  const int grid = (R + kSmallRowsPerCta - 1) / kSmallRowsPerCta;
  const TileArgs ta = tile_args(p, L, ws, T, p.E, true);
  const float* bias = p.cfg.use_bias ? p.w.bias : nullptr;
  float* sg = p.cfg.has_shared_gate ? reinterpret_cast<float*>(ws + L.sgate) : nullptr;
  const int vpl = (E + 31) / 32;
#define MOE_SMALL_CASE(V)                                                                          \
  do {                                                                                             \
    static bool done[64] = {};                                                                     \
    st = set_smem_attr(reinterpret_cast<const void*>(route_small_kernel<V>), 200 * 1024, done);    \
    if (st != cudaSuccess) return st;                                                              \
    MOE_PDL(route_small_kernel<V>, dim3(grid), dim3(256), smem, s, x, p.w.norm_w, p.w.router_w,   \
            bias, T, p.H, E, R, K, p.cfg.score_func, p.cfg.norm_topk_prob,                         \
            p.cfg.routed_scaling_factor, p.cfg.rms_norm_eps, reinterpret_cast<float*>(ws + L.logits), \
            reinterpret_cast<float*>(ws + L.rms), counter, reinterpret_cast<int32_t*>(ws + L.ids),  \
            reinterpret_cast<float*>(ws + L.wts), sg, reinterpret_cast<int32_t*>(ws + L.offsets),   \
            reinterpret_cast<int32_t*>(ws + L.perm), reinterpret_cast<int32_t*>(ws + L.slot_row), ta); \
  } while (0)
  if (vpl <= 1) MOE_SMALL_CASE(1);
  else if (vpl <= 2) MOE_SMALL_CASE(2);
  else if (vpl <= 4) MOE_SMALL_CASE(4);
  else if (vpl <= 8) MOE_SMALL_CASE(8);
  else if (vpl <= 16) MOE_SMALL_CASE(16);
  else MOE_SMALL_CASE(32);
#undef MOE_SMALL_CASE
  return cudaGetLastError();
}

cudaError_t launch_route(const Plan& p, const WsLayout& L, char* ws, const float* x, int T,
                         bool dispatch, cudaStream_t s, __half* xg_out) {
  const bool tc = route_uses_tc_router(p, T);
  cudaError_t st;
  if (route_uses_small(p, T)) {
    st = launch_route_small(p, L, ws, x, T, s);
    if (st != cudaSuccess || !dispatch) return st;
    const int rows = T * p.K + (p.SI > 0 ? T : 0);
    MOE_PDL(dispatch_kernel, dim3(min(rows, p.num_sms * 8)), dim3(256), 0, s,
            x, p.w.norm_w, reinterpret_cast<const float*>(ws + L.rms),
            reinterpret_cast<const int32_t*>(ws + L.perm), T, p.K, p.H, p.SI > 0,
            xg_out ? xg_out : reinterpret_cast<__half*>(ws + L.xg), reinterpret_cast<__half*>(ws + L.h16));
    return cudaGetLastError();
  }
  if (tc) {
    MOE_PDL(router_prep_kernel, dim3(T), dim3(256), 0, s, x, p.w.norm_w, p.H, p.cfg.rms_norm_eps,
                                         reinterpret_cast<float*>(ws + L.rms),
                                         reinterpret_cast<__half*>(ws + L.h16), p.d_err);
    st = cudaGetLastError();
    if (st != cudaSuccess) return st;
    st = launch_router_gemm(p, L, ws, T, s);
  } else {
    st = (router_bt(T) == 16) ? run_router<16>(p, L, ws, x, T, s) : run_router<64>(p, L, ws, x, T, s);
  }
  if (st != cudaSuccess) return st;
  const int E = p.E, K = p.K, R = p.router_rows;
  float* logits = reinterpret_cast<float*>(ws + L.logits);
  const float* bias = p.cfg.use_bias ? p.w.bias : nullptr;
  float* sg = p.cfg.has_shared_gate ? reinterpret_cast<float*>(ws + L.sgate) : nullptr;
  int32_t* ids = reinterpret_cast<int32_t*>(ws + L.ids);
  float* wts = reinterpret_cast<float*>(ws + L.wts);
  int32_t* offsets = reinterpret_cast<int32_t*>(ws + L.offsets);
  int32_t* perm = reinterpret_cast<int32_t*>(ws + L.perm);
  int32_t* slot_row = reinterpret_cast<int32_t*>(ws + L.slot_row);
  const TileArgs ta = tile_args(p, L, ws, T, p.E, true);
  const int vpl = (E + 31) / 32;
  if (route_uses_tail(p, T)) {
    const int words = (T + 31) / 32;
    const size_t smem = (static_cast<size_t>(T) * K + static_cast<size_t>(E) * words +
                         static_cast<size_t>(E)) * sizeof(int);
#define MOE_TAIL_CASE(V)                                                                        \
  do {                                                                                          \
    static bool done[64] = {};                                                                  \
    st = set_smem_attr(reinterpret_cast<const void*>(route_tail_kernel<V>), 160 * 1024, done);  \
    if (st != cudaSuccess) return st;                                                           \
    MOE_PDL(route_tail_kernel<V>, dim3(1), dim3(1024), smem, s, logits, bias, T, E, R, K, p.cfg.score_func,      \
                                               p.cfg.norm_topk_prob,                            \
                                               p.cfg.routed_scaling_factor, ids, wts, sg,       \
                                               offsets, perm, slot_row, ta);                    \
  } while (0)
    if (vpl <= 1) MOE_TAIL_CASE(1);
    else if (vpl <= 2) MOE_TAIL_CASE(2);
    else if (vpl <= 4) MOE_TAIL_CASE(4);
    else if (vpl <= 8) MOE_TAIL_CASE(8);
    else if (vpl <= 16) MOE_TAIL_CASE(16);
    else MOE_TAIL_CASE(32);
#undef MOE_TAIL_CASE
  } else {
    const int grid = (T + 7) / 8;
#define MOE_TOPK_CASE(V)                                                                        \
  do {                                                                                          \
    if (tc) {                                                                                   \
      int32_t* cand = reinterpret_cast<int32_t*>(ws + L.cand);                                  \
      int32_t* nrows = reinterpret_cast<int32_t*>(ws + L.ncand);                                \
      MOE_PDL(route_cand_kernel<V>, dim3(grid), dim3(256), 0, s, logits, router_tc_splits(p, T), bias, cand,     \
                                                nrows, T, E, R, K, p.cfg.score_func, p.d_err);  \
      MOE_PDL(route_exact_kernel, dim3(T), dim3(256), static_cast<size_t>(p.H) * 4, s, logits, cand, nrows, x, \
              p.w.norm_w, p.w.router_w,                                                                \
                                           reinterpret_cast<const float*>(ws + L.rms),          \
                                           reinterpret_cast<float*>(ws + L.exact), T, E, R, p.H, \
                                           p.cfg.has_shared_gate);                              \
      MOE_PDL(route_final_kernel<V>, dim3(grid), dim3(256), 0, s,                                                \
          logits, cand, nrows, reinterpret_cast<const float*>(ws + L.exact), bias, ids, wts, sg, \
          T, E, R, K, p.cfg.score_func, p.cfg.norm_topk_prob, p.cfg.routed_scaling_factor,     \
          p.d_err);                                                                             \
    } else                                                                                      \
      MOE_PDL(topk_kernel<V>, dim3(grid), dim3(256), 0, s, logits, bias, ids, wts, sg, T, E, R, K,               \
                                          p.cfg.score_func, p.cfg.norm_topk_prob,               \
                                          p.cfg.routed_scaling_factor, p.d_err);                \
  } while (0)
    if (vpl <= 1) MOE_TOPK_CASE(1);
    else if (vpl <= 2) MOE_TOPK_CASE(2);
    else if (vpl <= 4) MOE_TOPK_CASE(4);
    else if (vpl <= 8) MOE_TOPK_CASE(8);
    else if (vpl <= 16) MOE_TOPK_CASE(16);
    else MOE_TOPK_CASE(32);
#undef MOE_TOPK_CASE
    st = cudaGetLastError();
    if (st != cudaSuccess) return st;
    uint32_t* bmg = reinterpret_cast<uint32_t*>(ws + L.bm);
    int32_t* hist = reinterpret_cast<int32_t*>(ws + L.hist);
    int32_t* base = reinterpret_cast<int32_t*>(ws + L.base);
    static bool done_hist[64] = {};
    st = set_smem_attr(reinterpret_cast<const void*>(perm_hist_kernel), 1024 * 32 * sizeof(uint32_t),
                       done_hist);
    if (st != cudaSuccess) return st;
    MOE_PDL(perm_hist_kernel, dim3(L.nchunks), dim3(1024), static_cast<size_t>(E) * 32 * sizeof(uint32_t), s, 
        ids, T, K, E, K, 0, 0, bmg, hist, p.d_err);
    st = cudaGetLastError();
    if (st != cudaSuccess) return st;
    MOE_PDL(perm_scan_kernel, dim3(1), dim3(1024), 0, s, hist, L.nchunks, base, offsets, ta);
    st = cudaGetLastError();
    if (st != cudaSuccess) return st;
    const int entries = T * K;
    MOE_PDL(perm_scatter_kernel, dim3(min((entries + 255) / 256, p.num_sms * 8)), dim3(256), 0, s, 
        ids, bmg, base, T, K, E, K, 0, perm, slot_row);
  }
  st = cudaGetLastError();
  if (st != cudaSuccess || !dispatch) return st;
  if (tc) {  // h16 already holds the normalised rows: gather them per slot
    MOE_PDL(gather_rows_kernel, dim3(min(T * K, p.num_sms * 16)), dim3(256), 0, s, 
        reinterpret_cast<const __half*>(ws + L.h16), perm, T * K, p.H, p.H, K, nullptr,
        xg_out ? xg_out : reinterpret_cast<__half*>(ws + L.xg));
    return cudaGetLastError();
  }
  const int rows = T * K + (p.SI > 0 ? T : 0);
  MOE_PDL(dispatch_kernel, dim3(min(rows, p.num_sms * 8)), dim3(256), 0, s, 
      x, p.w.norm_w, reinterpret_cast<const float*>(ws + L.rms), perm, T, K, p.H, p.SI > 0,
      xg_out ? xg_out : reinterpret_cast<__half*>(ws + L.xg), reinterpret_cast<__half*>(ws + L.h16));
  return cudaGetLastError();
}

// ------------------------------------------------------------------ expert-parallel helpers
cudaError_t launch_group_rows(const Plan& p, const WsLayout& L, char* ws, const RowKeys& k,
                              const __half* rows, int row_ld, int n, cudaStream_t s) {
  const int E = p.n_local;
  uint32_t* bmg = reinterpret_cast<uint32_t*>(ws + L.bm);
  int32_t* hist = reinterpret_cast<int32_t*>(ws + L.hist);
  int32_t* base = reinterpret_cast<int32_t*>(ws + L.base);
  int32_t* offsets = reinterpret_cast<int32_t*>(ws + L.offsets);
  int32_t* perm = reinterpret_cast<int32_t*>(ws + L.perm);
  int32_t* slot_row = reinterpret_cast<int32_t*>(ws + L.slot_row);
  const TileArgs ta = tile_args(p, L, ws, 0, E, false);
  static bool done_hist[64] = {};
  cudaError_t st = set_smem_attr(reinterpret_cast<const void*>(perm_hist_kernel),
                                 1024 * 32 * sizeof(uint32_t), done_hist);
  if (st != cudaSuccess) return st;
  if (n > 0) {
    MOE_PDL(perm_hist_kernel, dim3(L.nchunks), dim3(1024), static_cast<size_t>(E) * 32 * sizeof(uint32_t), s, 
        k.keys, n, k.per_row, E, k.key_ld, k.key_base, k.pad_mode, bmg, hist, p.d_err);
    st = cudaGetLastError();
    if (st != cudaSuccess) return st;
  }
  MOE_PDL(perm_scan_kernel, dim3(1), dim3(1024), 0, s, hist, L.nchunks, base, offsets, ta);
  st = cudaGetLastError();
  if (st != cudaSuccess || n == 0) return st;
  const int slots = n * k.per_row;
  MOE_PDL(perm_scatter_kernel, dim3(min((slots + 255) / 256, p.num_sms * 8)), dim3(256), 0, s,
          k.keys, bmg, base, n, k.per_row, E, k.key_ld, k.key_base, perm, slot_row);
  st = cudaGetLastError();
  if (st != cudaSuccess) return st;
  MOE_PDL(gather_rows_kernel, dim3(min(slots, p.num_sms * 8)), dim3(256), 0, s, rows, perm, slots,
          p.H, row_ld, k.per_row, k.pad_mode ? offsets + E : nullptr,
          reinterpret_cast<__half*>(ws + L.xg));
  return cudaGetLastError();
}

cudaError_t launch_ep_pack(const Plan& p, const WsLayout& L, char* ws, const float* x, int T,
                           int cap, __half* send, cudaStream_t s) {
  // T == 0: every row is unused (the kernel reads nothing of the workspace)
  const bool tc = T > 0 && route_uses_tc_router(p, T);
  const int world = p.E / p.n_local;
  const int with_shared = (T > 0 && !tc && p.SI > 0) ? 1 : 0;
  const int rows = world * cap + (with_shared ? T : 0);
  auto at = [&](size_t off) { return T > 0 ? ws + off : nullptr; };
  MOE_PDL(ep_pack_kernel, dim3(min(rows, p.num_sms * 8)), dim3(256), 0, s, x, p.w.norm_w,
          reinterpret_cast<const float*>(at(L.rms)),
          tc ? reinterpret_cast<const __half*>(at(L.h16)) : nullptr,
          reinterpret_cast<const int32_t*>(at(L.perm)), reinterpret_cast<const int32_t*>(at(L.ids)),
          reinterpret_cast<const int32_t*>(at(L.offsets)), T, p.K, p.H, p.n_local, world, cap,
          with_shared, send, reinterpret_cast<int32_t*>(at(L.slot_row)),
          reinterpret_cast<__half*>(at(L.h16)), p.d_err);
  return cudaGetLastError();
}

int ep_token_row_halves(const Plan& p) { return p.H + ((4 * p.K + 7) & ~7); }

cudaError_t launch_ep_token_pack(const Plan& p, const WsLayout& L, char* ws, const float* x, int T,
                                 int cap, __half* send, cudaStream_t s) {
  const bool tc = T > 0 && route_uses_tc_router(p, T);
  const int with_shared = (T > 0 && !tc && p.SI > 0) ? 1 : 0;
  auto at = [&](size_t off) { return T > 0 ? ws + off : nullptr; };
  MOE_PDL(ep_token_pack_kernel, dim3(min(cap, p.num_sms * 8)), dim3(256), 0, s, x, p.w.norm_w,
          reinterpret_cast<const float*>(at(L.rms)),
          tc ? reinterpret_cast<const __half*>(at(L.h16)) : nullptr,
          reinterpret_cast<const int32_t*>(at(L.ids)), reinterpret_cast<const float*>(at(L.wts)),
          T, p.K, p.H, ep_token_row_halves(p), cap, with_shared, send,
          reinterpret_cast<__half*>(at(L.h16)));
  return cudaGetLastError();
}

cudaError_t launch_shared_tiles(const Plan& p, const WsLayout& L, char* ws, int T, cudaStream_t s) {
  const TileArgs ta = tile_args(p, L, ws, T, 0, true);
  MOE_PDL(perm_scan_kernel, dim3(1), dim3(1024), 0, s, nullptr, 0, nullptr, reinterpret_cast<int32_t*>(ws + L.offsets),
                                      ta);
  return cudaGetLastError();
}

}  // namespace moe
