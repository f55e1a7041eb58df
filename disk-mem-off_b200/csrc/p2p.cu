// Token-replicated expert-parallel exchange over peer memory (no collective library).
//
// The same data flow as the NCCL all-gather / reduce-scatter form of the exchange
// (see ep_token_pack_kernel and ep_partial_kernel), but the kernels that produce
// the data store it straight into the other GPUs' buffers over NVLink, mapped
// into this process with CUDA IPC, and publish an epoch flag there when a
// launch's stores are complete:
//
//   p2p_pack_kernel     token records of this rank -> every rank's receive slot
//                       [rank*cap, (rank+1)*cap); flag "records" [rank] = epoch
//   p2p_wait_kernel     wait (bounded) until every rank's flag reaches the epoch
//   (grouped GEMMs on the local receive buffer, as moe_ep_experts_gathered)
//   p2p_partial_kernel  fp32 partial sum of each received record -> its owner's
//                       partial slot [rank][i]; flag "partials" [rank] = epoch
//   p2p_wait_kernel
//   p2p_combine_kernel  x + sum over source ranks (rank order) + shared expert
//
// Each rank's buffers: receive [world*cap][ld] f16, partials [world][cap][H] fp32,
// flags [2][world] int32 (records, partials), all written only by the kernels
// above.  A rank cannot overwrite a buffer its peer still reads: a rank packs
// epoch e + 1 only after it has seen every peer's partials of epoch e, which each
// peer publishes after its last read of the epoch-e records, and it stores the
// partials of e + 1 only after seeing every peer's records of e + 1, which each
// peer packs after its combine of epoch e.
#include "common.cuh"
#include "moe_internal.h"

namespace moe {

// Publish `epoch` in slot `rank` of every rank's flag row `row` (system scope,
// release: the caller's stores, fenced before, are visible first).
MOE_DEV void publish_epoch(const P2PPeers& peers, int world, int row, int rank, int epoch) {
  for (int d = 0; d < world; ++d) {
    int* f = peers.flags[d] + row * world + rank;
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(f), "r"(epoch) : "memory");
  }
}

// Every CTA fences its stores system-wide and counts itself; the last one to
// arrive publishes the epoch and re-arms the counter for the next launch.
MOE_DEV void last_cta_publish(int* done, const P2PPeers& peers, int world, int row, int rank,
                              int epoch) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0 && threadIdx.y == 0) {
    const int nblocks = gridDim.x * gridDim.y;
    if (atomicAdd(done, 1) == nblocks - 1) {
      *done = 0;
      __threadfence_system();
      publish_epoch(peers, world, row, rank, epoch);
    }
  }
}

// One CTA per token record (as ep_token_pack_kernel), each 16-byte chunk stored to
// every rank's receive buffer at row rank * cap + t.
__global__ void __launch_bounds__(256) p2p_pack_kernel(
    const float* __restrict__ x, const float* __restrict__ wn, const float* __restrict__ rms,
    const __half* __restrict__ h16src, const int32_t* __restrict__ ids,
    const float* __restrict__ wts, int T, int K, int H, int ld, int cap, int with_shared,
    __half* __restrict__ h16, int rank, int world, P2PPeers peers, int epoch, int* done) {
  pdl_enter();
  const int tail_words = (ld - H) / 2;  // int32 words after the values
  for (int t = blockIdx.x; t < cap; t += gridDim.x) {
    const size_t row = static_cast<size_t>(rank) * cap + t;
    for (int i = threadIdx.x; i < tail_words; i += blockDim.x) {
      int32_t v = 0;
      if (i < K) {
        v = t < T ? ids[static_cast<size_t>(t) * K + i] : -1;
      } else if (i < 2 * K && t < T) {
        v = __float_as_int(wts[static_cast<size_t>(t) * K + (i - K)]);
      }
      for (int d = 0; d < world; ++d)
        reinterpret_cast<int32_t*>(static_cast<__half*>(peers.recv[d]) + row * ld + H)[i] = v;
    }
    if (t >= T) continue;
    const float inv = h16src ? 0.f : 1.0f / rms[t];
    const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(t) * H);
    const float4* wr = reinterpret_cast<const float4*>(wn);
    for (int v = threadIdx.x; v < (H >> 3); v += blockDim.x) {
      uint4 chunk;
      if (h16src) {
        chunk = reinterpret_cast<const uint4*>(h16src + static_cast<size_t>(t) * H)[v];
      } else {
        const float4 a0 = xr[2 * v], a1 = xr[2 * v + 1];
        const float4 g0 = wr[2 * v], g1 = wr[2 * v + 1];
        __half2 o[4];
        o[0] = __floats2half2_rn(g0.x * (a0.x * inv), g0.y * (a0.y * inv));
        o[1] = __floats2half2_rn(g0.z * (a0.z * inv), g0.w * (a0.w * inv));
        o[2] = __floats2half2_rn(g1.x * (a1.x * inv), g1.y * (a1.y * inv));
        o[3] = __floats2half2_rn(g1.z * (a1.z * inv), g1.w * (a1.w * inv));
        chunk = *reinterpret_cast<uint4*>(o);
        if (with_shared) reinterpret_cast<uint4*>(h16 + static_cast<size_t>(t) * H)[v] = chunk;
      }
      for (int d = 0; d < world; ++d)
        reinterpret_cast<uint4*>(static_cast<__half*>(peers.recv[d]) + row * ld)[v] = chunk;
    }
  }
  last_cta_publish(done, peers, world, 0, rank, epoch);
}

// Wait until flags[0 .. world) all reach `epoch` (one lane per rank, system-scope
// acquire loads), giving up after `limit` cycles with DEV_TIMEOUT_PEER.
__global__ void p2p_wait_kernel(const int* flags, int world, int epoch, long long limit, int* err) {
  pdl_enter();
  const int lane = threadIdx.x;
  bool ok = true;
  if (lane < world) {
    const long long start = clock64();
    while (true) {
      int v;
      asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(flags + lane) : "memory");
      if (v >= epoch) break;
      if (clock64() - start > limit) {
        ok = false;
        break;
      }
      __nanosleep(64);
    }
  }
  if (!__all_sync(0xffffffffu, ok) && lane == 0) record_error(err, DEV_TIMEOUT_PEER);
}

// The partial sum of received record t (ep_partial_kernel's arithmetic) goes to
// its owner o = t / cap, slot [rank][t % cap] of o's partial buffer.
__global__ void __launch_bounds__(256) p2p_partial_kernel(
    const __half* __restrict__ rows, int ld, int cap, const __half* __restrict__ y,
    const int32_t* __restrict__ slot_row, int K, int H, int e_begin, int e_loc, int rank, int world,
    P2PPeers peers, int epoch, int* done) {
  pdl_enter();
  const int n = world * cap;
  const int v = blockIdx.x * blockDim.x + threadIdx.x;  // float4 index
  if (v < (H >> 2)) {
    for (int t = blockIdx.y; t < n; t += gridDim.y) {
      const int32_t* tid = reinterpret_cast<const int32_t*>(rows + static_cast<size_t>(t) * ld + H);
      const float* tw = reinterpret_cast<const float*>(tid + K);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int j = 0; j < K; ++j) {
        const int e = tid[j] - e_begin;
        if (e < 0 || e >= e_loc) continue;
        const float w = tw[j];
        const uint2 raw = reinterpret_cast<const uint2*>(
            y + static_cast<size_t>(slot_row[t * K + j]) * H)[v];
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
        acc.x = __fadd_rn(acc.x, __fmul_rn(w, a.x));
        acc.y = __fadd_rn(acc.y, __fmul_rn(w, a.y));
        acc.z = __fadd_rn(acc.z, __fmul_rn(w, b.x));
        acc.w = __fadd_rn(acc.w, __fmul_rn(w, b.y));
      }
      const int o = t / cap, i = t - o * cap;
      float* dst = peers.part[o] + (static_cast<size_t>(rank) * cap + i) * H;
      reinterpret_cast<float4*>(dst)[v] = acc;
    }
  }
  last_cta_publish(done, peers, world, 1, rank, epoch);
}

// out = x + (sum over source ranks, in rank order, of their partials + shared).
__global__ void __launch_bounds__(256) p2p_combine_kernel(
    const float* __restrict__ x, const float* __restrict__ part, int cap, int world,
    const float* __restrict__ y_s, const float* __restrict__ sgate, float* __restrict__ out, int H) {
  pdl_enter();
  const int t = blockIdx.y;
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= (H >> 2)) return;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s = 0; s < world; ++s) {
    const float4 pv = reinterpret_cast<const float4*>(part + (static_cast<size_t>(s) * cap + t) * H)[v];
    acc.x = __fadd_rn(acc.x, pv.x);
    acc.y = __fadd_rn(acc.y, pv.y);
    acc.z = __fadd_rn(acc.z, pv.z);
    acc.w = __fadd_rn(acc.w, pv.w);
  }
  const size_t ro = static_cast<size_t>(t) * H;
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

// ------------------------------------------------------------------ launchers
cudaError_t launch_p2p_pack(const Plan& p, const WsLayout& L, char* ws, const float* x, int T,
                            int cap, int rank, int world, const P2PPeers& peers, int epoch,
                            int* done, cudaStream_t s) {
  const bool tc = T > 0 && route_uses_tc_router(p, T);
  const int with_shared = (T > 0 && !tc && p.SI > 0) ? 1 : 0;
  auto at = [&](size_t off) { return T > 0 ? ws + off : nullptr; };
  MOE_PDL(p2p_pack_kernel, dim3(max(1, min(cap, p.num_sms * 8))), dim3(256), 0, s, x, p.w.norm_w,
          reinterpret_cast<const float*>(at(L.rms)),
          tc ? reinterpret_cast<const __half*>(at(L.h16)) : nullptr,
          reinterpret_cast<const int32_t*>(at(L.ids)), reinterpret_cast<const float*>(at(L.wts)),
          T, p.K, p.H, ep_token_row_halves(p), cap, with_shared, reinterpret_cast<__half*>(at(L.h16)),
          rank, world, peers, epoch, done);
  return cudaGetLastError();
}

cudaError_t launch_p2p_wait(const int* flags, int world, int epoch, long long limit, int* err,
                            cudaStream_t s) {
  MOE_PDL(p2p_wait_kernel, dim3(1), dim3(32), 0, s, flags, world, epoch, limit, err);
  return cudaGetLastError();
}

cudaError_t launch_p2p_partial(const Plan& p, const __half* rows, int cap, const __half* y,
                               const int32_t* slot_row, int rank, int world, const P2PPeers& peers,
                               int epoch, int* done, cudaStream_t s) {
  const int nv = p.H >> 2;
  dim3 grid((nv + 255) / 256, min(world * cap, 65535));
  MOE_PDL(p2p_partial_kernel, grid, dim3(256), 0, s, rows, ep_token_row_halves(p), cap, y, slot_row,
          p.K, p.H, p.e_begin, p.n_local, rank, world, peers, epoch, done);
  return cudaGetLastError();
}

cudaError_t launch_p2p_combine(const Plan& p, const float* x, const float* part, int cap, int world,
                               const float* y_s, const float* sgate, float* out, int T,
                               cudaStream_t s) {
  const int nv = p.H >> 2;
  dim3 grid((nv + 255) / 256, T);
  MOE_PDL(p2p_combine_kernel, grid, dim3(256), 0, s, x, part, cap, world, p.SI > 0 ? y_s : nullptr,
          p.cfg.has_shared_gate ? sgate : nullptr, out, p.H);
  return cudaGetLastError();
}

}  // namespace moe
