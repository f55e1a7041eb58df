// Weighted combine + shared expert + residual (K5/K6 epilogue of the MoE block).
//
// Reference: glm4_moe.py:226-240 / qwen3_next.py:315-333
//   output[tok] += w_e * expert_out        (one term per selected expert)
//   output = output + shared_out           (shared_out * sigmoid(h . w_gate) on Qwen3)
//   return x + output
// Here the K routed terms of a token are summed in slot order (descending
// router weight) from the expert-major y rows, products and sums rounded
// separately like the reference's numpy expressions.  Deterministic: no atomics.
#include "common.cuh"
#include "moe_internal.h"

namespace moe {

// Expert rows are f16: written so by the down GEMM (single GPU) or returned over
// the expert-parallel exchange.
MOE_DEV float4 load_row4(const __half* y, size_t row, int H, int v) {
  const uint2 raw = reinterpret_cast<const uint2*>(y + row * H)[v];
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

template <typename YT>
__global__ void __launch_bounds__(256) combine_kernel(
    const float* __restrict__ x, const YT* __restrict__ y, const float* __restrict__ y_s,
    const int32_t* __restrict__ slot_row, const float* __restrict__ wts,
    const float* __restrict__ sgate, float* __restrict__ out, int K, int H) {
  pdl_enter();
  const int t = blockIdx.y;
  const int v = blockIdx.x * blockDim.x + threadIdx.x;  // float4 index
  if (v >= (H >> 2)) return;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j = 0; j < K; ++j) {
    const int row = slot_row[t * K + j];
    const float w = wts[t * K + j];
    const float4 yv = load_row4(y, static_cast<size_t>(row), H, v);
    acc.x = __fadd_rn(acc.x, __fmul_rn(w, yv.x));
    acc.y = __fadd_rn(acc.y, __fmul_rn(w, yv.y));
    acc.z = __fadd_rn(acc.z, __fmul_rn(w, yv.z));
    acc.w = __fadd_rn(acc.w, __fmul_rn(w, yv.w));
  }
  if (y_s) {
    float4 sv = reinterpret_cast<const float4*>(y_s + static_cast<size_t>(t) * H)[v];
    if (sgate) {
      const float g = sgate[t];
      sv.x = __fmul_rn(sv.x, g);
      sv.y = __fmul_rn(sv.y, g);
      sv.z = __fmul_rn(sv.z, g);
      sv.w = __fmul_rn(sv.w, g);
    }
    acc.x = __fadd_rn(acc.x, sv.x);
    acc.y = __fadd_rn(acc.y, sv.y);
    acc.z = __fadd_rn(acc.z, sv.z);
    acc.w = __fadd_rn(acc.w, sv.w);
  }
  const float4 xv = reinterpret_cast<const float4*>(x + static_cast<size_t>(t) * H)[v];
  float4 o;
  o.x = __fadd_rn(xv.x, acc.x);
  o.y = __fadd_rn(xv.y, acc.y);
  o.z = __fadd_rn(xv.z, acc.z);
  o.w = __fadd_rn(xv.w, acc.w);
  reinterpret_cast<float4*>(out + static_cast<size_t>(t) * H)[v] = o;
}

cudaError_t launch_combine_half(const Plan& p, const float* x, const __half* y, const float* y_s,
                                const int32_t* slot_row, const float* wts, const float* sgate,
                                float* out, int T, cudaStream_t s) {
  const int nv = p.H >> 2;
  dim3 grid((nv + 255) / 256, T);
  MOE_PDL(combine_kernel<__half>, dim3(grid), dim3(256), 0, s, x, y, p.SI > 0 ? y_s : nullptr, slot_row, wts,
                                              p.cfg.has_shared_gate ? sgate : nullptr, out, p.K,
                                              p.H);
  return cudaGetLastError();
}

// Token-replicated exchange, expert side: one fp32 partial sum per gathered
// token record over the slots whose expert is resident here (slot order, rounded
// like combine_kernel); zero for a record without one, so that the sum over
// ranks (a reduce-scatter) adds each routed term exactly once.
__global__ void __launch_bounds__(256) ep_partial_kernel(
    const __half* __restrict__ rows, int ld, int n, const __half* __restrict__ y,
    const int32_t* __restrict__ slot_row, float* __restrict__ partial, int K, int H, int e_begin,
    int e_loc) {
  pdl_enter();
  const int v = blockIdx.x * blockDim.x + threadIdx.x;  // float4 index
  if (v >= (H >> 2)) return;
  for (int t = blockIdx.y; t < n; t += gridDim.y) {
    const int32_t* tid = reinterpret_cast<const int32_t*>(rows + static_cast<size_t>(t) * ld + H);
    const float* tw = reinterpret_cast<const float*>(tid + K);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < K; ++j) {
      const int e = tid[j] - e_begin;
      if (e < 0 || e >= e_loc) continue;
      const float w = tw[j];
      const float4 yv = load_row4(y, static_cast<size_t>(slot_row[t * K + j]), H, v);
      acc.x = __fadd_rn(acc.x, __fmul_rn(w, yv.x));
      acc.y = __fadd_rn(acc.y, __fmul_rn(w, yv.y));
      acc.z = __fadd_rn(acc.z, __fmul_rn(w, yv.z));
      acc.w = __fadd_rn(acc.w, __fmul_rn(w, yv.w));
    }
    reinterpret_cast<float4*>(partial + static_cast<size_t>(t) * H)[v] = acc;
  }
}

cudaError_t launch_ep_partial(const Plan& p, const __half* rows, int n, const __half* y,
                              const int32_t* slot_row, float* partial, cudaStream_t s) {
  const int nv = p.H >> 2;
  dim3 grid((nv + 255) / 256, min(n, 65535));
  MOE_PDL(ep_partial_kernel, grid, dim3(256), 0, s, rows, ep_token_row_halves(p), n, y, slot_row,
          partial, p.K, p.H, p.e_begin, p.n_local);
  return cudaGetLastError();
}

// Combine of the token-replicated exchange: out = x + (partial + shared), partial
// being the routed sum that the reduce-scatter returned.
__global__ void __launch_bounds__(256) combine_partial_kernel(
    const float* __restrict__ x, const float* __restrict__ partial, const float* __restrict__ y_s,
    const float* __restrict__ sgate, float* __restrict__ out, int H) {
  pdl_enter();
  const int t = blockIdx.y;
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= (H >> 2)) return;
  const size_t ro = static_cast<size_t>(t) * H;
  float4 acc = reinterpret_cast<const float4*>(partial + ro)[v];
  if (y_s) {
    float4 sv = reinterpret_cast<const float4*>(y_s + ro)[v];
    if (sgate) {
      const float g = sgate[t];
      sv.x = __fmul_rn(sv.x, g);
      sv.y = __fmul_rn(sv.y, g);
      sv.z = __fmul_rn(sv.z, g);
      sv.w = __fmul_rn(sv.w, g);
    }
    acc.x = __fadd_rn(acc.x, sv.x);
    acc.y = __fadd_rn(acc.y, sv.y);
    acc.z = __fadd_rn(acc.z, sv.z);
    acc.w = __fadd_rn(acc.w, sv.w);
  }
  const float4 xv = reinterpret_cast<const float4*>(x + ro)[v];
  float4 o;
  o.x = __fadd_rn(xv.x, acc.x);
  o.y = __fadd_rn(xv.y, acc.y);
  o.z = __fadd_rn(xv.z, acc.z);
  o.w = __fadd_rn(xv.w, acc.w);
  reinterpret_cast<float4*>(out + ro)[v] = o;
}

cudaError_t launch_combine_partial(const Plan& p, const float* x, const float* partial,
                                   const float* y_s, const float* sgate, float* out, int T,
                                   cudaStream_t s) {
  const int nv = p.H >> 2;
  dim3 grid((nv + 255) / 256, T);
  MOE_PDL(combine_partial_kernel, grid, dim3(256), 0, s, x, partial, p.SI > 0 ? y_s : nullptr,
          p.cfg.has_shared_gate ? sgate : nullptr, out, p.H);
  return cudaGetLastError();
}

// Expert-parallel send metadata: the local expert id (on its owner rank) of every
// send row, and where each destination rank's rows start.
__global__ void ep_meta_kernel(const int32_t* __restrict__ perm, const int32_t* __restrict__ ids,
                               const int32_t* __restrict__ offsets, int n, int e_loc, int world,
                               int E, int32_t* __restrict__ send_experts,
                               int32_t* __restrict__ send_offsets) {
  pdl_enter();
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < n; r += gridDim.x * blockDim.x)
    send_experts[r] = ids[perm[r]] % e_loc;
  if (blockIdx.x == 0)
    for (int d = threadIdx.x; d <= world; d += blockDim.x) send_offsets[d] = offsets[min(d * e_loc, E)];
}

cudaError_t launch_ep_meta(const Plan& p, const int32_t* perm, const int32_t* ids,
                           const int32_t* offsets, int n, int32_t* send_experts,
                           int32_t* send_offsets, cudaStream_t s) {
  const int world = p.E / p.n_local;
  MOE_PDL(ep_meta_kernel, dim3(max(1, min((n + 255) / 256, p.num_sms * 4))), dim3(256), 0, s, 
      perm, ids, offsets, n, p.n_local, world, p.E, send_experts, send_offsets);
  return cudaGetLastError();
}

}  // namespace moe
