// GLM-4 MoE attention block on the device: replaces
// GLM4MoeExecutor._attention_block (offload_runtime/executors/glm4_moe.py:112-162),
// which the reference runs in NumPy after copying the whole layer back to the host:
//
//   h   = rms_norm(x, input_layernorm.weight)                      (launch_norm_rows)
//   qkv = h . [Wq; Wk; Wv]^T                  tcgen05 GEMM, fp32 K-split planes
//   q, k, v: + bias, per-head RMS norm * q_norm / k_norm, partial rotate-half
//            RoPE at positions 0..T-1                               (attn_qkv_kernel)
//   o   = softmax(q k^T / sqrt(d) + causal mask) v, GQA              (attn_fwd_kernel)
//   out = x + o . Wo^T                         tcgen05 GEMM planes + attn_out_kernel
//
// attn_fwd_kernel is a flash-attention kernel on the 5th-generation tensor cores:
// one CTA per (128-query tile, head); S = Q K^T and O += P V are tcgen05.mma with
// Q, K and V^T tiles in shared memory (by TMA), accumulators in TMEM, and P, the
// A operand of P V, written to TMEM by the softmax warps (two buffers).  Two
// softmax warpgroups split each query row's 128 keys (and O's columns) in halves
// and swap their partial row max through shared memory; they keep the max the
// exponentials refer to and the running sum in registers, and rescale O in TMEM
// only when the row max grows by more than 2^8 (in exp2 units), so most tiles
// neither rescale nor wait for the previous P V.  Keys arrive in 128-key tiles,
// K through a three-stage ring and V^T through a two-stage one, and S is
// computed two tiles ahead of the softmax.  All waits are bounded.
#include <math.h>

#include <algorithm>
#include <string>

#include "common.cuh"
#include "moe_internal.h"

namespace moe {

constexpr int kAttnTile = 128;  // queries per CTA and keys per tile

#define MOE_CUDA_RET(call)                  \
  do {                                      \
    const cudaError_t e_ = (call);          \
    if (e_ != cudaSuccess) return e_;       \
  } while (0)

struct AttnPlan {
  MoeAttnConfig cfg{};
  int H = 0, nh = 0, nkv = 0, hd = 0, rot = 0, nqkv = 0, nout = 0;
  int num_sms = 148;
  bool bound = false;
  bool has_bias = false;
  bool has_qk_norm = false;
  void* alloc = nullptr;
  size_t bytes = 0;
  __half* wqkv = nullptr;  // [nqkv][H] f16: q rows, then k rows, then v rows
  __half* wo = nullptr;    // [H][nh * hd] f16
  float* bqkv = nullptr;   // [nqkv] (zeros without bias)
  float* qn = nullptr;     // [hd] q_norm weight
  float* kn = nullptr;     // [hd] k_norm weight
  float* win = nullptr;    // [H] input_layernorm weight
  int* d_err = nullptr;
  CUtensorMap tm_qkv{}, tm_o{};
};

struct AttnWs {
  size_t rms, h16, qkv, rope, q, k, v, vt, o16, oplanes, total;
  int tpad, s1, s2;
};

static size_t a256(size_t v) { return (v + 255) & ~size_t(255); }

static AttnWs attn_ws(const AttnPlan& a, int T) {
  AttnWs w{};
  w.tpad = (T + kAttnTile - 1) / kAttnTile * kAttnTile;
  w.s1 = dense_gemm_splits(a.nqkv, T, a.H, a.num_sms);
  w.s2 = dense_gemm_splits(a.H, T, a.nout, a.num_sms);
  size_t o = 0;
  auto take = [&](size_t b) { const size_t at = o; o = a256(o + b); return at; };
  w.rms = take(static_cast<size_t>(T) * 4);
  w.h16 = take(static_cast<size_t>(T) * a.H * 2);
  w.qkv = take(static_cast<size_t>(w.s1) * T * a.nqkv * 4);
  w.rope = take(static_cast<size_t>(T) * (a.hd / 2) * 8);  // (cos, sin) per token and pair
  w.q = take(static_cast<size_t>(a.nh) * w.tpad * a.hd * 2);
  w.k = take(static_cast<size_t>(a.nkv) * w.tpad * a.hd * 2);
  w.v = take(static_cast<size_t>(a.nkv) * w.tpad * a.hd * 2);
  w.vt = take(static_cast<size_t>(a.nkv) * a.hd * w.tpad * 2);
  w.o16 = take(static_cast<size_t>(T) * a.nout * 2);
  w.oplanes = take(static_cast<size_t>(w.s2) * T * a.H * 4);
  w.total = o;
  return w;
}

// V consecutive floats (V = 2 or 4, 8- or 16-byte aligned) in one load
template <int V>
MOE_DEV void load_vec(const float* __restrict__ p, float (&out)[V]) {
  if constexpr (V == 4) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
  } else {
    const float2 a = *reinterpret_cast<const float2*>(p);
    out[0] = a.x; out[1] = a.y;
  }
}

// ------------------------------------------------------------------ q / k / v
// One CTA per (padded) token, a warp per head vector.  Sums the GEMM's K-split
// planes in split order, adds the bias, applies the per-head RMS norm
// (x / sqrt(mean(x^2) + eps) * w, _common.py:139-142) to q and k and the
// rotate-half RoPE (_common.py:106-126: frequencies theta^(-j / half) and angles
// in float64, angles rounded to float32) to their first `rot` dims, then writes
// q and k as f16 rows [head][tpad][hd] and v transposed [kv head][hd][tpad] (the
// K-major B operand of O += P V).  Rows past T are written as zeros.
template <int HD>
__global__ void __launch_bounds__(256) attn_qkv_kernel(
    const float* __restrict__ planes, int nsplit, int T, int tpad, int nh, int nkv,
    const float* __restrict__ bias, const float* __restrict__ qn, const float* __restrict__ kn,
    int rot, const float2* __restrict__ rope, float eps, __half* __restrict__ q16,
    __half* __restrict__ k16, __half* __restrict__ v16) {
  pdl_enter();
  constexpr int V = HD / 32;
  __shared__ float sh[8][HD];
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int heads = nh + 2 * nkv;
  const size_t nqkv = static_cast<size_t>(heads) * HD;
  const int half = rot / 2;
  // this token's rotation (cos, sin) pairs from attn_rope_kernel's table
  __shared__ float s_cos[HD / 2], s_sin[HD / 2];
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    const float2 cs = t < T ? rope[static_cast<size_t>(t) * half + j] : make_float2(1.f, 0.f);
    s_cos[j] = cs.x;
    s_sin[j] = cs.y;
  }
  __syncthreads();
  // one head per warp, two heads per pass with their loads issued together;
  // short sequences spread a token's heads over gridDim.y CTAs
  static_assert(V == 2 || V == 4, "head size 64 or 128");
  const int hstride = 8 * gridDim.y;
  const size_t trow = static_cast<size_t>(t < T ? t : 0) * nqkv;  // rows t >= T stay zero
  for (int hh0 = blockIdx.y * 8 + warp; hh0 < heads; hh0 += 2 * hstride) {
    float vv[2][V];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int hu = min(hh0 + u * hstride, heads - 1);
      const float* src = planes + trow + hu * HD + lane * V;
      if constexpr (V == 4) {
        const float4 a4 = *reinterpret_cast<const float4*>(src);
        vv[u][0] = a4.x; vv[u][1] = a4.y; vv[u][2] = a4.z; vv[u][3] = a4.w;
      } else {
        const float2 a2 = *reinterpret_cast<const float2*>(src);
        vv[u][0] = a2.x; vv[u][1] = a2.y;
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int hu = min(hh0 + u * hstride, heads - 1);
      for (int s = 1; s < nsplit; ++s) {  // split planes added in order
        const float* src = planes + static_cast<size_t>(s) * T * nqkv + trow + hu * HD + lane * V;
        if constexpr (V == 4) {
          const float4 a4 = *reinterpret_cast<const float4*>(src);
          vv[u][0] += a4.x; vv[u][1] += a4.y; vv[u][2] += a4.z; vv[u][3] += a4.w;
        } else {
          const float2 a2 = *reinterpret_cast<const float2*>(src);
          vv[u][0] += a2.x; vv[u][1] += a2.y;
        }
      }
      float bb[V];
      load_vec<V>(bias + hu * HD + lane * V, bb);
#pragma unroll
      for (int i = 0; i < V; ++i) vv[u][i] = t < T ? vv[u][i] + bb[i] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int hh = hh0 + u * hstride;
      if (hh >= heads) break;
      float* v = vv[u];
      const int kind = hh < nh ? 0 : (hh < nh + nkv ? 1 : 2);  // q, k, v
      if (t < T && kind < 2) {
        const float* nw = kind == 0 ? qn : kn;
        if (nw) {
          float ss = 0.f;
#pragma unroll
          for (int i = 0; i < V; ++i) ss = fmaf(v[i], v[i], ss);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
          const float rinv = 1.0f / sqrtf(ss / static_cast<float>(HD) + eps);
          float w[V];
          load_vec<V>(nw + lane * V, w);
#pragma unroll
          for (int i = 0; i < V; ++i) v[i] = (v[i] * rinv) * w[i];
        }
        if (half > 0) {
          // rotate-half partner of dim d (d +- half): with half a multiple of V and
          // half / V a power of two it sits in lane lane ^ (half / V), same slot
          const int pl = half / V;
          float pv[V];
          if (half % V == 0 && (pl & (pl - 1)) == 0 && 2 * pl <= 32) {
#pragma unroll
            for (int i = 0; i < V; ++i) pv[i] = __shfl_xor_sync(0xffffffffu, v[i], pl);
          } else {
#pragma unroll
            for (int i = 0; i < V; ++i) sh[warp][lane * V + i] = v[i];
            __syncwarp();
#pragma unroll
            for (int i = 0; i < V; ++i) {
              const int d = lane * V + i;
              pv[i] = d < rot ? sh[warp][d < half ? d + half : d - half] : 0.f;
            }
            __syncwarp();
          }
#pragma unroll
          for (int i = 0; i < V; ++i) {
            const int d = lane * V + i;
            if (d < rot) {
              const int j = d < half ? d : d - half;
              const float c = s_cos[j], sn = s_sin[j];
              v[i] = d < half ? v[i] * c - pv[i] * sn : v[i] * c + pv[i] * sn;
            }
          }
        }
      }
      // q, k and v rows [head][tpad][HD] (v is transposed by attn_vt_kernel)
      __half* dst = kind == 0 ? q16 + (static_cast<size_t>(hh) * tpad + t) * HD
                  : kind == 1 ? k16 + (static_cast<size_t>(hh - nh) * tpad + t) * HD
                              : v16 + (static_cast<size_t>(hh - nh - nkv) * tpad + t) * HD;
      __half2 h2[V / 2];
  #pragma unroll
      for (int i = 0; i < V / 2; ++i) h2[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
      if constexpr (V == 4) *reinterpret_cast<uint2*>(dst + lane * V) = *reinterpret_cast<uint2*>(h2);
      else *reinterpret_cast<uint32_t*>(dst + lane * V) = *reinterpret_cast<uint32_t*>(h2);
    }
  }
}

// RoPE table of positions 0..T-1: (cos, sin) of pair j of token t, computed as the
// reference does, in double precision: freq = 1 / theta^(j / half), angle =
// float(t * freq), then cos / sin of that angle.  One thread per (token, pair).
__global__ void __launch_bounds__(256) attn_rope_kernel(float2* __restrict__ rope, int T, int half,
                                                        float theta) {
  pdl_enter();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * half) return;
  const int t = i / half, j = i - t * half;
  const double freq = 1.0 / pow(static_cast<double>(theta),
                                static_cast<double>(j) / static_cast<double>(half));
  const float ang = static_cast<float>(static_cast<double>(t) * freq);
  rope[i] = make_float2(static_cast<float>(cos(static_cast<double>(ang))),
                        static_cast<float>(sin(static_cast<double>(ang))));
}

// v [kv head][tpad][HD] -> vt [kv head][HD][tpad] (the K-major B operand of P V),
// one 64 x 64 tile per CTA through shared memory.
__global__ void __launch_bounds__(256) attn_vt_kernel(const __half* __restrict__ v16,
                                                      __half* __restrict__ vt16, int tpad, int HD) {
  pdl_enter();
  __shared__ __align__(16) __half tile[64][64 + 8];
  const int t0 = blockIdx.x * 64, d0 = blockIdx.y * 64, h = blockIdx.z;
  const __half* src = v16 + (static_cast<size_t>(h) * tpad + t0) * HD + d0;
  for (int i = threadIdx.x; i < 64 * 8; i += blockDim.x) {  // 64 rows x 8 chunks of 8 halves
    const int r = i >> 3, c = (i & 7) * 8;
    const uint4 q = *reinterpret_cast<const uint4*>(src + static_cast<size_t>(r) * HD + c);
    const __half* qh = reinterpret_cast<const __half*>(&q);
#pragma unroll
    for (int e = 0; e < 8; ++e) tile[c + e][r] = qh[e];
  }
  __syncthreads();
  __half* dst = vt16 + (static_cast<size_t>(h) * HD + d0) * tpad + t0;
  for (int i = threadIdx.x; i < 64 * 8; i += blockDim.x) {
    const int r = i >> 3, c = (i & 7) * 8;
    *reinterpret_cast<uint4*>(dst + static_cast<size_t>(r) * tpad + c) =
        *reinterpret_cast<const uint4*>(&tile[r][c]);
  }
}

// ------------------------------------------------------------------ flash attention
template <int HD>
struct FaCfg {
  static constexpr int kQ = kAttnTile * HD * 2;        // Q tile: HD / 64 blocks of 16 KiB
  static constexpr int kK = kAttnTile * HD * 2;        // one K stage
  static constexpr int kVblk = HD * 128;               // one 64-key block of V^T (HD rows x 128 B)
  static constexpr int kV = 2 * kVblk;                 // one V^T stage (128 keys)
  static constexpr int kKStages = 3;                   // K tiles for S two tiles ahead
  static constexpr int kXch = 2 * 2 * kAttnTile * 4;   // row-max / row-sum exchange [2][2][128]
  // at least 120 KiB, so that one CTA holds an SM (and all 512 TMEM columns) for
  // either head size: a second CTA would only wait in tcgen05.alloc
  static constexpr size_t kUsed = 1024 + kQ + kKStages * kK + 2 * kV + 256 + kXch;
  static constexpr size_t kSmem = kUsed > 120 * 1024 ? kUsed : 120 * 1024;
  static constexpr uint32_t kTmemCols = 512;
  // TMEM columns: S[2] at 0 / 128 (f32), O at 256 (HD f32), P[2] at 384 / 448
  // (128 keys as f16 pairs, the A operand of P V)
  static constexpr uint32_t kOCol = 2 * kAttnTile;
  static constexpr uint32_t kPCol = 3 * kAttnTile;
  static constexpr uint32_t kPCols = kAttnTile / 2;
};

struct FaArgs {
  CUtensorMap tq, tk, tv;
  int T, tpad, nh, nkv, nqt;
  float scale_log2;  // log2(e) / sqrt(head_dim)
  __half* out16;     // [T][nh * HD]
  int* err;
};

// warps: 0 Q / K loads, 1 MMA issue, 2-9 softmax (two warpgroups: key columns
// 0-63 and 64-127), 10 V loads
constexpr int kFaSoftmaxThreads = 256;
constexpr int kFaThreads = 64 + kFaSoftmaxThreads + 32;

// 2^x on the special-function unit, subnormal results flushed to zero (P is
// rounded to f16 afterwards, whose smallest subnormal is 2^-24)
MOE_DEV float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int HD>
__global__ void __launch_bounds__(kFaThreads, 1) attn_fwd_kernel(const __grid_constant__ FaArgs args) {
  using C = FaCfg<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + C::kQ;
  uint8_t* sV = sK + C::kKStages * C::kK;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + 2 * C::kV);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;    // [kKStages] K ring (freed when S = Q K^T completes)
  uint64_t* k_empty = bars + 4;   // [kKStages]
  uint64_t* v_full = bars + 7;    // [2] V^T ring (freed when P V completes)
  uint64_t* v_empty = bars + 9;   // [2]
  uint64_t* s_full = bars + 11;   // [2]
  uint64_t* s_free = bars + 13;   // [2]
  uint64_t* p_full = bars + 15;   // [2] P buffer b written (tiles j with j % 2 == b)
  uint64_t* o_done = bars + 17;   // [2] P V of a tile on buffer b finished
  uint64_t* mma_done = bars + 19;
  uint64_t* xch_full = bars + 20; // [2] both halves' partial row max (row sum at the end) written
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 22);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* xch = reinterpret_cast<float*>(bars + 32);  // [parity][half][query row]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = args.nqt - 1 - static_cast<int>(blockIdx.x);  // long (late) tiles first
  const int h = blockIdx.y;
  const int kvh = h / (args.nh / args.nkv);
  const int q0 = qt * kAttnTile;
  const int nkt = qt + 1;  // causal: key tiles 0..qt

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    static_assert(C::kKStages == 3, "barrier slots");
    for (int b = 0; b < C::kKStages; ++b) {
      mbar_init(&k_full[b], 1);
      mbar_init(&k_empty[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&v_full[b], 1);
      mbar_init(&v_empty[b], 1);
      mbar_init(&s_full[b], 1);
      mbar_init(&s_free[b], kFaSoftmaxThreads);
      mbar_init(&p_full[b], kFaSoftmaxThreads);
      mbar_init(&o_done[b], 1);
      mbar_init(&xch_full[b], kFaSoftmaxThreads);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&args.tq);
    tma_prefetch_desc(&args.tk);
    tma_prefetch_desc(&args.tv);
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();

  if (warp == 0 || warp == 10) {
    // ------------------------------------------------------------ TMA producers
    // warp 0: Q, then K tiles; warp 10: V^T tiles.  A K stage is free as soon as
    // its S completes, so the next K tiles load while the softmax still runs.
    if (lane == 0) {
      const bool kside = warp == 0;
      if (kside) {
        mbar_arrive_expect_tx(q_full, C::kQ);
#pragma unroll
        for (int kb = 0; kb < HD / 64; ++kb)
          tma_load_2d(sQ + kb * 16384, &args.tq, kb * 64, h * args.tpad + q0, q_full);
      }
      uint64_t* full = kside ? k_full : v_full;
      uint64_t* empty = kside ? k_empty : v_empty;
      const int nst = kside ? C::kKStages : 2;
      int issued = 0;
      for (int j = 0; j < nkt; ++j) {
        const int s = j % nst;
        if (!mbar_wait_bounded(&empty[s], ((j / nst) & 1) ^ 1, abort_flag)) {
          *abort_flag = 1;
          record_error(args.err, DEV_TIMEOUT_EMPTY);
          break;
        }
        if (kside) {
          mbar_arrive_expect_tx(&full[s], C::kK);
#pragma unroll
          for (int kb = 0; kb < HD / 64; ++kb)
            tma_load_2d(sK + s * C::kK + kb * 16384, &args.tk, kb * 64, kvh * args.tpad + j * kAttnTile,
                        &full[s]);
        } else {
          mbar_arrive_expect_tx(&full[s], C::kV);
#pragma unroll
          for (int kb = 0; kb < 2; ++kb)
            tma_load_2d(sV + s * C::kV + kb * C::kVblk, &args.tv, j * kAttnTile + kb * 64, kvh * HD,
                        &full[s]);
        }
        issued = j + 1;
      }
      // every copy this thread started must land before the CTA exits
      if (kside) mbar_wait_drain(q_full, 0);
      for (int j = issued - 1; j >= 0 && j >= issued - nst; --j) mbar_wait_drain(&full[j % nst], (j / nst) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_s = idesc_f16_f32(kAttnTile, kAttnTile);
      const uint32_t idesc_o = idesc_f16_f32(kAttnTile, HD);
      const uint32_t aq = smem_u32(sQ), ak = smem_u32(sK), av = smem_u32(sV);
      bool ok = mbar_wait_bounded(q_full, 0, abort_flag);
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1, sk = j % C::kKStages;
        if (!mbar_wait_bounded(&k_full[sk], (j / C::kKStages) & 1, abort_flag)) return false;
        if (!mbar_wait_bounded(&s_free[s], ((j >> 1) & 1) ^ 1, abort_flag)) return false;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const int kb = k >> 2, kk = k & 3;
          tc_mma_f16(tmem_base + s * kAttnTile, sw128_desc(aq + kb * 16384 + kk * 32),
                     sw128_desc(ak + sk * C::kK + kb * 16384 + kk * 32), idesc_s, k > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[s]);
        tc_commit(&k_empty[sk]);
        return true;
      };
      // S runs two tiles ahead: S of tile j + 2 goes into tile j's buffer as soon as
      // the softmax has read it, ahead of P V of tile j
      if (ok) ok = issue_s(0);
      if (ok && nkt > 1) ok = issue_s(1);
      for (int j = 0; ok && j < nkt; ++j) {
        if (j + 2 < nkt && !issue_s(j + 2)) {
          ok = false;
          break;
        }
        const int s = j & 1;
        if (!mbar_wait_bounded(&p_full[j & 1], (j >> 1) & 1, abort_flag) ||
            !mbar_wait_bounded(&v_full[s], (j >> 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // O += P V with P (128 queries x 128 keys, f16) read from TMEM
        const uint32_t pa = tmem_base + C::kPCol + (j & 1) * C::kPCols;
#pragma unroll
        for (int k = 0; k < kAttnTile / 16; ++k) {
          const int kb = k >> 2, kk = k & 3;
          tc_mma_f16_ts(tmem_base + C::kOCol, pa + k * 8,
                        sw128_desc(av + s * C::kV + kb * C::kVblk + kk * 32), idesc_o,
                        (j > 0 || k > 0) ? 1u : 0u);
        }
        tc_commit(&o_done[j & 1]);
        tc_commit(&v_empty[s]);
      }
      if (!ok) {
        *abort_flag = 1;
        record_error(args.err, DEV_TIMEOUT_FULL);
      }
      tc_commit(mma_done);  // no MMA may still write TMEM when it is released
      mbar_wait_drain(mma_done, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax (warps 2-9)
    // warps 2-5 take key columns 0-63 and O columns [0, HD/2); warps 6-9 the other
    // halves; a warp reaches TMEM lanes 32 * (warp % 4) .. + 31, one query row each
    constexpr int kH = kAttnTile / 2;  // keys per half
    const int half = (warp - 2) >> 2;
    const int qrow = (warp & 3) * 32 + lane;
    const int qi = q0 + qrow;
    const uint32_t lbase = tmem_base + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t scol = half * kH;
    const uint32_t ocol = C::kOCol + half * (HD / 2);
    float* my_x = xch + half * kAttnTile + qrow;              // + parity * 2 * kAttnTile
    const float* peer_x = xch + (half ^ 1) * kAttnTile + qrow;
    // partner exchange of one float per row through shared memory, parity
    // buffered: tile j's values are overwritten only by tile j + 2's, which no
    // thread writes before both halves have read tile j + 1's
    auto exchange = [&](int j, float v, float* out) -> bool {
      my_x[(j & 1) * 2 * kAttnTile] = v;
      mbar_arrive(&xch_full[j & 1]);
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&xch_full[j & 1], (j >> 1) & 1, abort_flag)))
        return false;
      *out = peer_x[(j & 1) * 2 * kAttnTile];
      return true;
    };
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkt; ++j) {
      const int s = j & 1;
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&s_full[s], (j >> 1) & 1, abort_flag))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sc[kH];
#pragma unroll
      for (int c = 0; c < kH / 32; ++c) {
        float part[32];
        tmem_ld32(lbase + s * kAttnTile + scol + c * 32, part);
#pragma unroll
        for (int i = 0; i < 32; ++i) sc[c * 32 + i] = part[i];
      }
      // S is in registers: the MMA may overwrite this buffer with tile j + 2
      tc_fence_before();
      mbar_arrive(&s_free[s]);
      if (j == qt) {  // diagonal tile: keys after the query are masked (causal)
#pragma unroll
        for (int c = 0; c < kH; ++c)
          if (half * kH + c > qrow) sc[c] = -INFINITY;
      }
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < kH; ++c) mx4[c & 3] = fmaxf(mx4[c & 3], sc[c]);
      float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      float mx_peer;
      if (!exchange(j, mx, &mx_peer)) {
        ok = false;
        break;
      }
      mx = fmaxf(mx, mx_peer);
      // m is the max the exponentials in O and l refer to; it moves (and O and l are
      // rescaled) only when the row max grows by more than 2^8 in exp2 units, so
      // most tiles need neither the rescale nor to wait for the previous P V; P then
      // holds values up to 256, well inside f16.  Both halves of a row see the
      // same m, mx and so the same decision.
      const float m_cand = fmaxf(m, mx);  // finite: key 0 is never masked
      const bool grow = (m_cand - m) * args.scale_log2 > 8.f;  // always on the first tile
      float alpha = 1.f;
      if (grow) {
        alpha = exp2f((m - m_cand) * args.scale_log2);
        m = m_cand;
      }
      const float ms = m * args.scale_log2;
      float rs4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < kH; ++c) {
        sc[c] = ex2_ftz(fmaf(sc[c], args.scale_log2, -ms));
        rs4[c & 3] += sc[c];
      }
      l = l * alpha + ((rs4[0] + rs4[1]) + (rs4[2] + rs4[3]));
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
        // O must be complete up to tile j - 1 before it is rescaled
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1,
                                                       abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          float o[16];
          tmem_ld16(lbase + ocol + c * 16, o);
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] *= alpha;
          tmem_st16(lbase + ocol + c * 16, o);
        }
      }
      if (j >= 2) {
        // P buffer j % 2 is free once P V of tile j - 2 has finished
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&o_done[j & 1], ((j >> 1) & 1) ^ 1, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      // this half's 64 keys -> 32 TMEM columns of f16 pairs (even key in the low half)
      uint32_t pk[kH / 2];
#pragma unroll
      for (int i = 0; i < kH / 2; ++i) {
        const __half2 hp = __floats2half2_rn(sc[2 * i], sc[2 * i + 1]);
        pk[i] = *reinterpret_cast<const uint32_t*>(&hp);
      }
      tmem_st32_nowait(lbase + C::kPCol + (j & 1) * C::kPCols + half * (kH / 2), pk);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[j & 1]);
    }
    float l_peer = 0.f;
    if (ok && !exchange(nkt, l, &l_peer)) ok = false;
    if (ok && !__all_sync(0xffffffffu, mbar_wait_bounded(&o_done[(nkt - 1) & 1], ((nkt - 1) >> 1) & 1,
                                                          abort_flag)))
      ok = false;
    if (ok) {
      tc_fence_after();
      const float inv = 1.0f / (half == 0 ? l + l_peer : l_peer + l);
      const int ld = args.nh * HD;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        float o[16];
        tmem_ld16(lbase + ocol + c * 16, o);
        __half2 hv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) hv[i] = __floats2half2_rn(o[2 * i] * inv, o[2 * i + 1] * inv);
        if (qi < args.T) {
          uint4* dst = reinterpret_cast<uint4*>(args.out16 + static_cast<size_t>(qi) * ld + h * HD +
                                                half * (HD / 2) + c * 16);
          dst[0] = *reinterpret_cast<uint4*>(&hv[0]);
          dst[1] = *reinterpret_cast<uint4*>(&hv[4]);
        }
      }
    } else {
      *abort_flag = 1;
      record_error(args.err, DEV_TIMEOUT_TMEM_FULL);
    }
  }
  pdl_release();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// out = x + sum_s planes[s] (the o_proj K-split planes, added in split order)
__global__ void __launch_bounds__(256) attn_out_kernel(const float* __restrict__ x,
                                                       const float* __restrict__ planes, int nsplit,
                                                       size_t n, float* __restrict__ out) {
  pdl_enter();
  // n is a multiple of 4 (H is a multiple of 64): float4 at a time, planes in order
  const size_t n4 = n / 4;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < nsplit; ++s) {
      const float4 p = reinterpret_cast<const float4*>(planes + static_cast<size_t>(s) * n)[i];
      acc.x += p.x;
      acc.y += p.y;
      acc.z += p.z;
      acc.w += p.w;
    }
    const float4 xv = reinterpret_cast<const float4*>(x)[i];
    reinterpret_cast<float4*>(out)[i] = make_float4(xv.x + acc.x, xv.y + acc.y, xv.z + acc.z, xv.w + acc.w);
  }
}

template <int HD>
static cudaError_t attn_launch(const AttnPlan& a, const AttnWs& w, char* ws, const float* x,
                               float* out, int T, cudaStream_t s) {
  MOE_CUDA_RET(launch_norm_rows(x, a.win, a.H, a.cfg.rms_norm_eps, T,
                                reinterpret_cast<float*>(ws + w.rms),
                                reinterpret_cast<__half*>(ws + w.h16), a.d_err, s));
  MOE_CUDA_RET(launch_dense_gemm(a.tm_qkv, a.nqkv, a.H, reinterpret_cast<const __half*>(ws + w.h16), T,
                                 reinterpret_cast<float*>(ws + w.qkv), w.s1, a.d_err, a.num_sms, s));
  const int half = a.rot / 2;
  if (half > 0) {
    MOE_PDL(attn_rope_kernel, dim3((T * half + 255) / 256), dim3(256), 0, s,
            reinterpret_cast<float2*>(ws + w.rope), T, half, a.cfg.rope_theta);
  }
  // enough CTAs for every SM to hold several: one per token at long sequences, a
  // token's heads in groups of 8 across CTAs at short ones
  const int groups = (a.nh + 2 * a.nkv + 7) / 8;
  const int gy = std::max(1, std::min(groups, (8 * a.num_sms + w.tpad - 1) / w.tpad));
  MOE_PDL(attn_qkv_kernel<HD>, dim3(w.tpad, gy), dim3(256), 0, s, reinterpret_cast<const float*>(ws + w.qkv),
          w.s1, T, w.tpad, a.nh, a.nkv, a.bqkv, a.has_qk_norm ? a.qn : nullptr,
          a.has_qk_norm ? a.kn : nullptr, a.rot, reinterpret_cast<const float2*>(ws + w.rope),
          a.cfg.rms_norm_eps,
          reinterpret_cast<__half*>(ws + w.q), reinterpret_cast<__half*>(ws + w.k),
          reinterpret_cast<__half*>(ws + w.v));
  MOE_PDL(attn_vt_kernel, dim3(w.tpad / 64, HD / 64, a.nkv), dim3(256), 0, s,
          reinterpret_cast<const __half*>(ws + w.v), reinterpret_cast<__half*>(ws + w.vt), w.tpad, HD);
  FaArgs fa{};
  std::string err;
  if (!make_tmap_2d(&fa.tq, ws + w.q, false, HD, static_cast<uint64_t>(a.nh) * w.tpad, 64, kAttnTile,
                    true, &err) ||
      !make_tmap_2d(&fa.tk, ws + w.k, false, HD, static_cast<uint64_t>(a.nkv) * w.tpad, 64, kAttnTile,
                    true, &err) ||
      !make_tmap_2d(&fa.tv, ws + w.vt, false, w.tpad, static_cast<uint64_t>(a.nkv) * HD, 64, HD, true,
                    &err)) {
    set_error(err);
    return cudaErrorInvalidValue;
  }
  fa.T = T;
  fa.tpad = w.tpad;
  fa.nh = a.nh;
  fa.nkv = a.nkv;
  fa.nqt = w.tpad / kAttnTile;
  fa.scale_log2 = static_cast<float>(1.4426950408889634 / sqrt(static_cast<double>(HD)));
  fa.out16 = reinterpret_cast<__half*>(ws + w.o16);
  fa.err = a.d_err;
  constexpr size_t smem = FaCfg<HD>::kSmem;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    const cudaError_t st = cudaFuncSetAttribute(attn_fwd_kernel<HD>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(smem));
    if (st != cudaSuccess) return st;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  MOE_PDL(attn_fwd_kernel<HD>, dim3(fa.nqt, a.nh), dim3(kFaThreads), smem, s, fa);
  MOE_CUDA_RET(launch_dense_gemm(a.tm_o, a.H, a.nout, reinterpret_cast<const __half*>(ws + w.o16), T,
                                 reinterpret_cast<float*>(ws + w.oplanes), w.s2, a.d_err, a.num_sms, s));
  const size_t n = static_cast<size_t>(T) * a.H;
  const int grid = static_cast<int>(std::min<size_t>((n + 255) / 256, static_cast<size_t>(a.num_sms) * 8));
  MOE_PDL(attn_out_kernel, dim3(grid), dim3(256), 0, s, x, reinterpret_cast<const float*>(ws + w.oplanes),
          w.s2, n, out);
  return cudaSuccess;
}

}  // namespace moe

// ====================================================================== C ABI
using namespace moe;

struct MoeAttn {
  AttnPlan a;
};

namespace {

int afail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

#define MOE_ATT_CUDA(call)                                                               \
  do {                                                                                   \
    const cudaError_t st_ = (call);                                                      \
    if (st_ != cudaSuccess) return afail(MOE_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(st_)); \
  } while (0)

int parse_dtype_name(const char* d) {
  const std::string s(d ? d : "");
  if (s == "float32" || s == "<f4" || s == "f4") return SRC_F32;
  if (s == "float16" || s == "<f2" || s == "f2") return SRC_F16;
  if (s == "bfloat16" || s == "bf16") return SRC_BF16;
  return -1;
}

// the part of a tensor name after an optional "model.layers.N." prefix
std::string short_name(const char* n) {
  std::string s(n ? n : "");
  const size_t p = s.find("self_attn.");
  if (p != std::string::npos) return s.substr(p);
  const size_t q = s.find("input_layernorm.weight");
  if (q != std::string::npos) return s.substr(q);
  return s;
}

}  // namespace

extern "C" {

int moe_attn_create(const MoeAttnConfig* cfg, MoeAttn** out) {
  if (!cfg || !out) return afail(MOE_ERR_INVALID, "null argument");
  const MoeAttnConfig& c = *cfg;
  if (c.head_dim != 64 && c.head_dim != 128)
    return afail(MOE_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  if (c.heads <= 0 || c.kv_heads <= 0 || c.heads % c.kv_heads != 0)
    return afail(MOE_ERR_INVALID, "heads must be a positive multiple of kv_heads");
  if (c.hidden <= 0 || c.hidden % 64 != 0)
    return afail(MOE_ERR_UNSUPPORTED, "hidden must be a positive multiple of 64");
  if (c.rotary_dim < 0 || c.rotary_dim > c.head_dim || c.rotary_dim % 2 != 0)
    return afail(MOE_ERR_INVALID, "rotary_dim must be even and at most head_dim");
  if (c.max_tokens <= 0) return afail(MOE_ERR_INVALID, "max_tokens must be positive");
  if (!(c.rope_theta > 0.f)) return afail(MOE_ERR_INVALID, "rope_theta must be positive");
  MOE_ATT_CUDA(cudaSetDevice(c.device));
  MoeAttn* h = new MoeAttn();
  AttnPlan& a = h->a;
  a.cfg = c;
  a.H = c.hidden;
  a.nh = c.heads;
  a.nkv = c.kv_heads;
  a.hd = c.head_dim;
  a.rot = c.rotary_dim;
  a.nqkv = (a.nh + 2 * a.nkv) * a.hd;
  a.nout = a.nh * a.hd;
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, c.device);
  a.num_sms = sms > 0 ? sms : 148;
  cudaError_t st = cudaMalloc(&a.d_err, sizeof(int));
  if (st == cudaSuccess) st = cudaMemset(a.d_err, 0, sizeof(int));
  if (st != cudaSuccess) {
    delete h;
    return afail(MOE_ERR_CUDA, std::string("cudaMalloc(error word): ") + cudaGetErrorString(st));
  }
  *out = h;
  return MOE_OK;
}

int moe_attn_destroy(MoeAttn* h) {
  if (!h) return MOE_OK;
  cudaSetDevice(h->a.cfg.device);
  if (h->a.alloc) cudaFree(h->a.alloc);
  if (h->a.d_err) cudaFree(h->a.d_err);
  delete h;
  return MOE_OK;
}

uint64_t moe_attn_weight_bytes(const MoeAttn* h) { return h ? h->a.bytes : 0; }

int moe_attn_bind(MoeAttn* h, const void* blob_dev, uint64_t blob_bytes, const MoeTensorDesc* descs,
                  int32_t n_descs, void* stream) {
  if (!h || !blob_dev || !descs || n_descs <= 0) return afail(MOE_ERR_INVALID, "null argument");
  AttnPlan& a = h->a;
  MOE_ATT_CUDA(cudaSetDevice(a.cfg.device));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  struct Src {
    const char* ptr = nullptr;
    int dtype = -1;
  };
  Src wq, wk, wv, wo, bq, bk, bv, qn, kn, win;
  const char* base = static_cast<const char*>(blob_dev);
  const int H = a.H, nq = a.nh * a.hd, nk = a.nkv * a.hd, hd = a.hd;
  for (int i = 0; i < n_descs; ++i) {
    const MoeTensorDesc& d = descs[i];
    const std::string n = short_name(d.name);
    Src* dst = nullptr;
    int64_t rows = 0, cols = 1;
    if (n == "self_attn.q_proj.weight") { dst = &wq; rows = nq; cols = H; }
    else if (n == "self_attn.k_proj.weight") { dst = &wk; rows = nk; cols = H; }
    else if (n == "self_attn.v_proj.weight") { dst = &wv; rows = nk; cols = H; }
    else if (n == "self_attn.o_proj.weight") { dst = &wo; rows = H; cols = nq; }
    else if (n == "self_attn.q_proj.bias") { dst = &bq; rows = nq; }
    else if (n == "self_attn.k_proj.bias") { dst = &bk; rows = nk; }
    else if (n == "self_attn.v_proj.bias") { dst = &bv; rows = nk; }
    else if (n == "self_attn.q_norm.weight") { dst = &qn; rows = hd; }
    else if (n == "self_attn.k_norm.weight") { dst = &kn; rows = hd; }
    else if (n == "input_layernorm.weight") { dst = &win; rows = H; }
    if (!dst) continue;
    const int dt = parse_dtype_name(d.dtype);
    if (dt < 0) return afail(MOE_ERR_UNSUPPORTED, std::string("unsupported dtype for ") + d.name);
    const int64_t esz = dt == SRC_F32 ? 4 : 2;
    int64_t numel = 1;
    for (int k = 0; k < d.ndim && k < 2; ++k) numel *= d.shape[k];
    const bool shape_ok = (cols == 1) ? (numel == rows) : (d.ndim == 2 && d.shape[0] == rows && d.shape[1] == cols);
    if (!shape_ok || numel * esz != d.nbytes)
      return afail(MOE_ERR_INVALID, std::string("shape / nbytes mismatch for ") + d.name);
    if (d.offset < 0 || static_cast<uint64_t>(d.offset + d.nbytes) > blob_bytes)
      return afail(MOE_ERR_INVALID, std::string("tensor outside the blob: ") + d.name);
    *dst = Src{base + d.offset, dt};
  }
  if (!wq.ptr) return afail(MOE_ERR_MISSING_TENSOR, "self_attn.q_proj.weight");
  if (!wk.ptr) return afail(MOE_ERR_MISSING_TENSOR, "self_attn.k_proj.weight");
  if (!wv.ptr) return afail(MOE_ERR_MISSING_TENSOR, "self_attn.v_proj.weight");
  if (!wo.ptr) return afail(MOE_ERR_MISSING_TENSOR, "self_attn.o_proj.weight");
  if (!win.ptr) return afail(MOE_ERR_MISSING_TENSOR, "input_layernorm.weight");
  if ((qn.ptr != nullptr) != (kn.ptr != nullptr))
    return afail(MOE_ERR_MISSING_TENSOR, "q_norm and k_norm come as a pair");
  size_t o = 0;
  auto take = [&](size_t b) { const size_t at = o; o = a256(o + b); return at; };
  const size_t o_wqkv = take(static_cast<size_t>(a.nqkv) * H * 2);
  const size_t o_wo = take(static_cast<size_t>(H) * a.nout * 2);
  const size_t o_b = take(static_cast<size_t>(a.nqkv) * 4);
  const size_t o_qn = take(static_cast<size_t>(hd) * 4);
  const size_t o_kn = take(static_cast<size_t>(hd) * 4);
  const size_t o_win = take(static_cast<size_t>(H) * 4);
  const size_t o_flag = take(16);
  if (!a.alloc) {
    MOE_ATT_CUDA(cudaMalloc(&a.alloc, o));
    a.bytes = o;
  }
  char* wb = static_cast<char*>(a.alloc);
  a.wqkv = reinterpret_cast<__half*>(wb + o_wqkv);
  a.wo = reinterpret_cast<__half*>(wb + o_wo);
  a.bqkv = reinterpret_cast<float*>(wb + o_b);
  a.qn = reinterpret_cast<float*>(wb + o_qn);
  a.kn = reinterpret_cast<float*>(wb + o_kn);
  a.win = reinterpret_cast<float*>(wb + o_win);
  int* range_err = reinterpret_cast<int*>(wb + o_flag);
  MOE_ATT_CUDA(cudaMemsetAsync(range_err, 0, sizeof(int), s));
  MOE_ATT_CUDA(cudaMemsetAsync(a.bqkv, 0, static_cast<size_t>(a.nqkv) * 4, s));
  MOE_ATT_CUDA(launch_pack_rows(wq.ptr, wq.dtype, a.wqkv, false, nullptr, nq, H, range_err, s));
  MOE_ATT_CUDA(launch_pack_rows(wk.ptr, wk.dtype, a.wqkv + static_cast<size_t>(nq) * H, false, nullptr, nk, H,
                                range_err, s));
  MOE_ATT_CUDA(launch_pack_rows(wv.ptr, wv.dtype, a.wqkv + static_cast<size_t>(nq + nk) * H, false, nullptr,
                                nk, H, range_err, s));
  MOE_ATT_CUDA(launch_pack_rows(wo.ptr, wo.dtype, a.wo, false, nullptr, H, nq, range_err, s));
  if (bq.ptr) MOE_ATT_CUDA(launch_to_f32(bq.ptr, bq.dtype, a.bqkv, nq, s));
  if (bk.ptr) MOE_ATT_CUDA(launch_to_f32(bk.ptr, bk.dtype, a.bqkv + nq, nk, s));
  if (bv.ptr) MOE_ATT_CUDA(launch_to_f32(bv.ptr, bv.dtype, a.bqkv + nq + nk, nk, s));
  if (qn.ptr) {
    MOE_ATT_CUDA(launch_to_f32(qn.ptr, qn.dtype, a.qn, hd, s));
    MOE_ATT_CUDA(launch_to_f32(kn.ptr, kn.dtype, a.kn, hd, s));
  }
  MOE_ATT_CUDA(launch_to_f32(win.ptr, win.dtype, a.win, H, s));
  int h_range = 0;
  MOE_ATT_CUDA(cudaMemcpyAsync(&h_range, range_err, sizeof(int), cudaMemcpyDeviceToHost, s));
  MOE_ATT_CUDA(cudaStreamSynchronize(s));
  if (h_range) return afail(MOE_ERR_RANGE, "an attention weight does not fit f16 (|w| > 65504)");
  a.has_bias = bq.ptr || bk.ptr || bv.ptr;
  a.has_qk_norm = qn.ptr != nullptr;
  std::string err;
  if (!make_tmap_2d(&a.tm_qkv, a.wqkv, false, H, a.nqkv, kBK, kBM, true, &err) ||
      !make_tmap_2d(&a.tm_o, a.wo, false, a.nout, H, kBK, kBM, true, &err))
    return afail(MOE_ERR_CUDA, err);
  a.bound = true;
  return MOE_OK;
}

uint64_t moe_attn_workspace_bytes(const MoeAttn* h, int32_t T) {
  if (!h || T <= 0) return 0;
  return attn_ws(h->a, T).total;
}

int moe_attn_forward(MoeAttn* h, const float* x_dev, float* out_dev, int32_t T, void* workspace,
                     uint64_t workspace_bytes, void* stream) {
  if (!h) return afail(MOE_ERR_INVALID, "null attention plan");
  AttnPlan& a = h->a;
  if (!a.bound) return afail(MOE_ERR_NOT_BOUND, "moe_attn_bind has not been called");
  if (T < 0 || T > a.cfg.max_tokens) return afail(MOE_ERR_INVALID, "T outside [0, max_tokens]");
  if (T == 0) return MOE_OK;
  if (!x_dev || !out_dev) return afail(MOE_ERR_INVALID, "null x / out");
  if (x_dev == out_dev) return afail(MOE_ERR_INVALID, "x and out may not alias");
  if (misaligned16(x_dev) || misaligned16(out_dev))
    return afail(MOE_ERR_INVALID, "x and out must be 16-byte aligned");
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return afail(MOE_ERR_WORKSPACE, "workspace must be a 256-byte aligned device pointer");
  const AttnWs w = attn_ws(a, T);
  if (workspace_bytes < w.total) return afail(MOE_ERR_WORKSPACE, "workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  const cudaError_t st = a.hd == 128 ? attn_launch<128>(a, w, ws, x_dev, out_dev, T, s)
                                     : attn_launch<64>(a, w, ws, x_dev, out_dev, T, s);
  if (st != cudaSuccess) return afail(MOE_ERR_CUDA, std::string("attention launch: ") + cudaGetErrorString(st));
  return MOE_OK;
}

int moe_attn_status(MoeAttn* h, void* stream) {
  if (!h) return afail(MOE_ERR_INVALID, "null attention plan");
  AttnPlan& a = h->a;
  MOE_ATT_CUDA(cudaSetDevice(a.cfg.device));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int v = 0;
  MOE_ATT_CUDA(cudaMemcpyAsync(&v, a.d_err, sizeof(int), cudaMemcpyDeviceToHost, s));
  MOE_ATT_CUDA(cudaMemsetAsync(a.d_err, 0, sizeof(int), s));
  MOE_ATT_CUDA(cudaStreamSynchronize(s));
  if (v == DEV_OK) return MOE_OK;
  if (v >= DEV_TIMEOUT_FULL && v <= DEV_TIMEOUT_CONV)
    return afail(MOE_ERR_TIMEOUT, "an attention wait ran out of time (code " + std::to_string(v) + ")");
  return afail(MOE_ERR_DEVICE, "an attention kernel reported device error code " + std::to_string(v));
}

}  // extern "C"
