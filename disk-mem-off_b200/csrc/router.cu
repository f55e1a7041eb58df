// Router, top-k and token permutation kernels (K1/K2 of the MoE block).
//
// Reference arithmetic (disk-mem-off, offload_runtime/executors):
//   rms_norm      _common.py:73-75       h = w * (x / sqrt(mean(x^2) + eps))
//   router        glm4_moe.py:181-183    logits = h @ Wg^T (+ e_score_correction_bias)
//   scoring/top-k glm4_moe.py:185-200    softmax, top-k by prob, renormalise, * scale
//                 qwen3_next.py:278-293  (no bias, no scale)
//   dispatch      glm4_moe.py:206-215    per expert, tokens ascending
// Everything on the routing path stays fp32.  Ranking uses the biased logit
// (softmax is monotone in it), exact ties go to the lower expert id.
#include <float.h>

#include "common.cuh"
#include "moe_internal.h"

namespace moe {

// ------------------------------------------------------------------ RMSNorm
// One CTA per token: h32 (router input, fp32) and h16 (expert GEMM operand).
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float* __restrict__ x,
                                                      const float* __restrict__ w,
                                                      float* __restrict__ h32,
                                                      __half* __restrict__ h16, int H,
                                                      float eps) {
  const int t = blockIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(t) * H);
  const int nv = H >> 2;
  float ss = 0.f;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    float4 v = xr[i];
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
  }
  __shared__ float red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float rms = sqrtf(red[0] / static_cast<float>(H) + eps);
  const float4* wr = reinterpret_cast<const float4*>(w);
  float4* o32 = reinterpret_cast<float4*>(h32 + static_cast<size_t>(t) * H);
  __half2* o16 = reinterpret_cast<__half2*>(h16 + static_cast<size_t>(t) * H);
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    float4 v = xr[i];
    float4 g = wr[i];
    float4 r;
    r.x = g.x * (v.x / rms);
    r.y = g.y * (v.y / rms);
    r.z = g.z * (v.z / rms);
    r.w = g.w * (v.w / rms);
    o32[i] = r;
    o16[2 * i] = __floats2half2_rn(r.x, r.y);
    o16[2 * i + 1] = __floats2half2_rn(r.z, r.w);
  }
}

// ------------------------------------------------------------------ router
// logits = h32 @ Wr^T in fp32, split along K.  CTA (rx, s, ty) computes router
// rows [32 rx, 32 rx + 32) x tokens [BT ty, BT ty + BT) over its K range, in
// chunks of 128: the whole chunk of both operands is requested with cp.async at
// once (so a decode step pays one memory latency, not one per k-step), then
// each thread accumulates TPT x EPT outputs reading float4s along K.  Partial
// sums go to part[s][t][r]; the top-k kernel adds the S slices in order s = 0..S-1,
// so the result is deterministic.
constexpr int kRouterKc = 128;      // K elements per chunk
constexpr int kRouterRows = 32;     // router rows per CTA
constexpr int kRouterPad = 4;       // smem row padding (floats)

MOE_DEV void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}

template <int BT>
__global__ void __launch_bounds__(256) router_splitk_kernel(const float* __restrict__ h32,
                                                            const float* __restrict__ wr,
                                                            float* __restrict__ part, int T,
                                                            int H, int R, int k_per_split) {
  constexpr int EPT = (BT == 64) ? 4 : 2;     // router rows per thread
  constexpr int XT = kRouterRows / EPT;       // threads along rows
  constexpr int YT = 256 / XT;                // threads along tokens
  constexpr int TPT = BT / YT;                // tokens per thread
  constexpr int LD = kRouterKc + kRouterPad;  // smem row stride (floats)
  extern __shared__ __align__(16) float rsm[];
  float* hs = rsm;                 // [BT][LD]
  float* ws = rsm + BT * LD;       // [32][LD]
  const int r0 = blockIdx.x * kRouterRows;
  const int t0 = blockIdx.z * BT;
  const int kb = blockIdx.y * k_per_split;
  const int ke = min(H, kb + k_per_split);
  const int tid = threadIdx.x;
  const int ty = tid / XT, tx = tid % XT;
  float acc[TPT][EPT] = {};
  for (int k0 = kb; k0 < ke; k0 += kRouterKc) {
    const int kn = min(kRouterKc, ke - k0);  // multiple of 16 (H % 16 == 0)
    const int nv = kn >> 2;                  // float4 per row in this chunk
    for (int i = tid; i < BT * (kRouterKc / 4); i += 256) {
      const int row = i / (kRouterKc / 4), v = i % (kRouterKc / 4);
      float* dst = hs + row * LD + v * 4;
      if (t0 + row < T && v < nv) cp_async16(dst, h32 + static_cast<size_t>(t0 + row) * H + k0 + v * 4);
      else *reinterpret_cast<float4*>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int i = tid; i < kRouterRows * (kRouterKc / 4); i += 256) {
      const int row = i / (kRouterKc / 4), v = i % (kRouterKc / 4);
      float* dst = ws + row * LD + v * 4;
      if (r0 + row < R && v < nv) cp_async16(dst, wr + static_cast<size_t>(r0 + row) * H + k0 + v * 4);
      else *reinterpret_cast<float4*>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    __syncthreads();
#pragma unroll 4
    for (int k = 0; k < kRouterKc; k += 4) {
      float4 a[TPT], b[EPT];
#pragma unroll
      for (int i = 0; i < TPT; ++i) a[i] = *reinterpret_cast<const float4*>(hs + (ty + YT * i) * LD + k);
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
  float* out = part + static_cast<size_t>(blockIdx.y) * T * R;
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
}

// ------------------------------------------------------------------ top-k
// One warp per token.  Lane l holds experts l, l+32, ...  Scores are ranked by
// (key desc, id asc); weights follow the reference formulas in fp32.
template <int VPL>
__global__ void __launch_bounds__(256) topk_kernel(const float* __restrict__ part,
                                                   const float* __restrict__ bias,
                                                   int32_t* __restrict__ ids_out,
                                                   float* __restrict__ w_out,
                                                   float* __restrict__ sgate, int T, int E,
                                                   int R, int K, int nsplit, int score_func,
                                                   int norm, float scale, int* err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= T) return;
  // logit of router row r for this token: split-K partials added in split order
  auto logit = [&](int r) {
    const float* p = part + static_cast<size_t>(t) * R + r;
    float v = p[0];
    for (int q = 1; q < nsplit; ++q) v += p[static_cast<size_t>(q) * T * R];
    return v;
  };
  float key[VPL], val[VPL];
  float m = -FLT_MAX;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int e = j * 32 + lane;
    key[j] = -FLT_MAX;
    val[j] = 0.f;
    if (e < E) {
      float l = logit(e);
      if (score_func == MOE_SCORE_SOFTMAX) {
        if (bias) l = l + bias[e];
        key[j] = l;
        val[j] = l;
        m = fmaxf(m, l);
      } else {
        const float s = sigmoid_f(l);
        val[j] = s;
        key[j] = bias ? s + bias[e] : s;
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
      const int e = j * 32 + lane;
      if (e < E) {
        val[j] = expf(val[j] - m);
        s += val[j];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    denom = s;
  }
  // iterative arg-max selection; `taken` marks this lane's retired experts
  int sel_id[kMaxTopK];
  float sel_w[kMaxTopK];
  uint32_t taken = 0u;
  for (int r = 0; r < K; ++r) {
    float bk = -FLT_MAX;
    int bid = 0x7fffffff;
    float bv = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int e = j * 32 + lane;
      if (e < E && !((taken >> j) & 1u) &&
          (bid == 0x7fffffff || key[j] > bk || (key[j] == bk && e < bid))) {
        bk = key[j];
        bid = e;
        bv = val[j];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ok = __shfl_xor_sync(0xffffffffu, bk, o);
      const int oid = __shfl_xor_sync(0xffffffffu, bid, o);
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      if (oid != 0x7fffffff &&
          (bid == 0x7fffffff || ok > bk || (ok == bk && oid < bid))) {
        bk = ok;
        bid = oid;
        bv = ov;
      }
    }
    if (bid >= E) {  // K > E cannot happen for a validated plan
      record_error(err, DEV_BAD_ROUTE);
      bid = 0;
    }
    sel_id[r] = bid;
    sel_w[r] = (score_func == MOE_SCORE_SOFTMAX) ? bv / denom : bv;
    if ((bid & 31) == lane) taken |= 1u << (bid >> 5);
  }
  if (lane == 0) {
    float sum = 0.f;
    if (norm)
      for (int r = 0; r < K; ++r) sum += sel_w[r];
    for (int r = 0; r < K; ++r) {
      float wv = sel_w[r];
      if (norm) wv = wv / (sum + 1e-20f);
      wv = wv * scale;
      ids_out[static_cast<size_t>(t) * K + r] = sel_id[r];
      w_out[static_cast<size_t>(t) * K + r] = wv;
    }
    if (sgate) sgate[t] = sigmoid_f(logit(E));
  }
}

// ------------------------------------------------------------------ permutation
// Per chunk of 1024 tokens: a bitmask per expert (bit = token has the expert in
// its top-k).  Counts are popcounts; the rank of a token inside its expert is
// the popcount of the lower bits, so the dispatch order (tokens ascending
// inside an expert) is deterministic without any ordering of atomics.
__global__ void __launch_bounds__(1024) perm_hist_kernel(const int32_t* __restrict__ ids, int T,
                                                         int K, int E, uint32_t* __restrict__ bmg,
                                                         int32_t* __restrict__ hist, int* err) {
  extern __shared__ uint32_t bm[];  // [E][32]
  const int c = blockIdx.x;
  const int tbeg = c * kPermChunk;
  const int tcnt = min(kPermChunk, T - tbeg);
  for (int i = threadIdx.x; i < E * 32; i += blockDim.x) bm[i] = 0u;
  __syncthreads();
  for (int q = threadIdx.x; q < tcnt * K; q += blockDim.x) {
    const int tl = q / K;
    const int e = ids[static_cast<size_t>(tbeg) * K + q];
    if (e < 0 || e >= E) {
      record_error(err, DEV_BAD_ROUTE);
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

// Single CTA: expert offsets, per-chunk bases and the two GEMM tile lists.
__global__ void __launch_bounds__(1024) perm_scan_kernel(
    const int32_t* __restrict__ hist, int nchunks, int E, int T, int bn, int mt1, int mt2,
    int mt1s, int has_shared, int max1, int max2, int32_t* __restrict__ base,
    int32_t* __restrict__ offsets, Tile* __restrict__ tiles1, Tile* __restrict__ tiles2,
    int32_t* __restrict__ tile_count, int* err) {
  const int e = threadIdx.x;
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
  const int ntile_n = (e < E) ? (tot + bn - 1) / bn : 0;
  int tot1 = 0, tot2 = 0;
  const int p1 = block_excl_scan(ntile_n * mt1, &tot1);
  const int p2 = block_excl_scan(ntile_n * mt2, &tot2);
  // tile lists: expert-major, m outer, token tiles inner (a weight tile is
  // reused by neighbouring CTAs while it is still in L2)
  if (e < E) {
    int q1 = p1, q2 = p2;
    for (int m = 0; m < mt1; ++m)
      for (int n = 0; n < ntile_n; ++n, ++q1)
        if (q1 < max1) tiles1[q1] = Tile{e, m * kBM, off + n * bn, min(bn, tot - n * bn)};
    for (int m = 0; m < mt2; ++m)
      for (int n = 0; n < ntile_n; ++n, ++q2)
        if (q2 < max2) tiles2[q2] = Tile{e, m * kBM, off + n * bn, min(bn, tot - n * bn)};
  }
  __syncthreads();
  const int nts = has_shared ? (T + bn - 1) / bn : 0;
  for (int i = threadIdx.x; i < mt1s * nts; i += blockDim.x) {
    const int m = i / nts, n = i % nts;
    if (tot1 + i < max1) tiles1[tot1 + i] = Tile{E, m * kBM, n * bn, min(bn, T - n * bn)};
  }
  for (int i = threadIdx.x; i < mt2 * nts; i += blockDim.x) {
    const int m = i / nts, n = i % nts;
    if (tot2 + i < max2) tiles2[tot2 + i] = Tile{E, m * kBM, n * bn, min(bn, T - n * bn)};
  }
  if (threadIdx.x == 0) {
    const int c1 = tot1 + mt1s * nts, c2 = tot2 + mt2 * nts;
    if (c1 > max1 || c2 > max2) record_error(err, DEV_BAD_TILE);
    tile_count[0] = min(c1, max1);
    tile_count[1] = min(c2, max2);
  }
}

// One warp per (token, slot): rank from the chunk bitmask, write perm /
// slot_row, and copy the token's f16 row into its dispatch slot.
__global__ void __launch_bounds__(256) perm_scatter_gather_kernel(
    const int32_t* __restrict__ ids, const uint32_t* __restrict__ bmg,
    const int32_t* __restrict__ base, const __half* __restrict__ h16, int T, int K, int E, int H,
    int32_t* __restrict__ perm, int32_t* __restrict__ slot_row, __half* __restrict__ xg) {
  const int lane = threadIdx.x & 31;
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  for (int q = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); q < T * K; q += nwarps) {
    const int t = q / K;
    const int e = ids[q];
    if (e < 0 || e >= E) continue;  // reported by perm_hist_kernel
    const int c = t / kPermChunk, tl = t % kPermChunk;
    const uint32_t word = bmg[(static_cast<size_t>(c) * E + e) * 32 + lane];
    int cnt = 0;
    if (lane < (tl >> 5)) cnt = __popc(word);
    else if (lane == (tl >> 5)) cnt = __popc(word & ((1u << (tl & 31)) - 1u));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    const int row = base[static_cast<size_t>(c) * E + e] + cnt;
    if (lane == 0) {
      perm[row] = q;
      slot_row[q] = row;
    }
    if (xg) {
      const uint4* src = reinterpret_cast<const uint4*>(h16 + static_cast<size_t>(t) * H);
      uint4* dst = reinterpret_cast<uint4*>(xg + static_cast<size_t>(row) * H);
      for (int v = lane; v < (H >> 3); v += 32) dst[v] = src[v];
    }
  }
}

// ------------------------------------------------------------------ launchers
cudaError_t launch_rmsnorm(const Plan& p, const float* x, float* h32, __half* h16, int T,
                           cudaStream_t s) {
  rmsnorm_kernel<<<T, 256, 0, s>>>(x, p.w.norm_w, h32, h16, p.H, p.cfg.rms_norm_eps);
  return cudaGetLastError();
}

int router_splits(const Plan& p, int T) {
  const int nchunks = (p.H + kRouterKc - 1) / kRouterKc;
  const int bt = T <= 16 ? 16 : 64;
  const int tiles = ((p.router_rows + kRouterRows - 1) / kRouterRows) * ((T + bt - 1) / bt);
  // enough CTAs to cover the SMs about twice, never more splits than K chunks
  int s = (2 * p.num_sms + tiles - 1) / tiles;
  if (s > nchunks) s = nchunks;
  return s < 1 ? 1 : s;
}

template <int BT>
static cudaError_t run_router(const Plan& p, const float* h32, float* part, int T, int S,
                              cudaStream_t s) {
  constexpr size_t smem = static_cast<size_t>(BT + kRouterRows) * (kRouterKc + kRouterPad) * sizeof(float);
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t a = cudaFuncSetAttribute(router_splitk_kernel<BT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (a != cudaSuccess) return a;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int nchunks = (p.H + kRouterKc - 1) / kRouterKc;
  const int k_per_split = ((nchunks + S - 1) / S) * kRouterKc;
  dim3 grid((p.router_rows + kRouterRows - 1) / kRouterRows, S, (T + BT - 1) / BT);
  router_splitk_kernel<BT><<<grid, 256, smem, s>>>(h32, p.w.router_w, part, T, p.H,
                                                    p.router_rows, k_per_split);
  return cudaGetLastError();
}

cudaError_t launch_router(const Plan& p, const float* h32, float* logits, int T,
                          cudaStream_t s) {
  const int S = router_splits(p, T);
  return T <= 16 ? run_router<16>(p, h32, logits, T, S, s) : run_router<64>(p, h32, logits, T, S, s);
}

cudaError_t launch_topk(const Plan& p, const float* logits, int32_t* ids, float* wts,
                        float* sgate, int T, cudaStream_t s) {
  const int E = p.E;
  const float* bias = p.cfg.use_bias ? p.w.bias : nullptr;
  float* sg = p.cfg.has_shared_gate ? sgate : nullptr;
  const int grid = (T + 7) / 8;
  const int nsplit = router_splits(p, T);
#define MOE_TOPK_CASE(V)                                                                     \
  topk_kernel<V><<<grid, 256, 0, s>>>(logits, bias, ids, wts, sg, T, E, p.router_rows, p.K,  \
                                      nsplit, p.cfg.score_func, p.cfg.norm_topk_prob,        \
                                      p.cfg.routed_scaling_factor, p.d_err)
  const int vpl = (E + 31) / 32;
  if (vpl <= 1) MOE_TOPK_CASE(1);
  else if (vpl <= 2) MOE_TOPK_CASE(2);
  else if (vpl <= 4) MOE_TOPK_CASE(4);
  else if (vpl <= 8) MOE_TOPK_CASE(8);
  else if (vpl <= 16) MOE_TOPK_CASE(16);
  else MOE_TOPK_CASE(32);
#undef MOE_TOPK_CASE
  return cudaGetLastError();
}

cudaError_t launch_permute(const Plan& p, const WsLayout& L, char* ws, const int32_t* ids,
                           const __half* h16, int T, cudaStream_t s) {
  const int E = p.E, K = p.K;
  uint32_t* bmg = reinterpret_cast<uint32_t*>(ws + L.bm);
  int32_t* hist = reinterpret_cast<int32_t*>(ws + L.hist);
  int32_t* base = reinterpret_cast<int32_t*>(ws + L.base);
  int32_t* offsets = reinterpret_cast<int32_t*>(ws + L.offsets);
  const size_t smem = static_cast<size_t>(E) * 32 * sizeof(uint32_t);
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t a = cudaFuncSetAttribute(perm_hist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         1024 * 32 * static_cast<int>(sizeof(uint32_t)));
    if (a != cudaSuccess) return a;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  perm_hist_kernel<<<L.nchunks, 1024, smem, s>>>(ids, T, K, E, bmg, hist, p.d_err);
  cudaError_t st = cudaGetLastError();
  if (st != cudaSuccess) return st;
  const int mt1 = (2 * p.I + kBM - 1) / kBM;
  const int mt2 = (p.H + kBM - 1) / kBM;
  const int mt1s = p.SI > 0 ? (2 * p.SI + kBM - 1) / kBM : 0;
  perm_scan_kernel<<<1, 1024, 0, s>>>(hist, L.nchunks, E, T, L.bn, mt1, mt2, mt1s, p.SI > 0,
                                      L.max_tiles1, L.max_tiles2, base, offsets,
                                      reinterpret_cast<Tile*>(ws + L.tiles1),
                                      reinterpret_cast<Tile*>(ws + L.tiles2),
                                      reinterpret_cast<int32_t*>(ws + L.tile_count), p.d_err);
  st = cudaGetLastError();
  if (st != cudaSuccess) return st;
  const int entries = T * K;
  const int grid = min((entries + 7) / 8, p.num_sms * 8);
  perm_scatter_gather_kernel<<<grid, 256, 0, s>>>(
      ids, bmg, base, h16, T, K, E, p.H, reinterpret_cast<int32_t*>(ws + L.perm),
      reinterpret_cast<int32_t*>(ws + L.slot_row),
      h16 ? reinterpret_cast<__half*>(ws + L.xg) : nullptr);
  return cudaGetLastError();
}

}  // namespace moe
