// Grouped expert GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces the per-expert fp32 BLAS calls of the reference
// (glm4_moe.py:218-224 and qwen3_next.py:307-313, shared expert 234-238 /
// 321-331) with one persistent launch per projection:
//
//   gate/up : D[2I rows of W13, tokens] = W13_e . X_e^T, epilogue silu(g) * u -> act (f16)
//   down    : D[H rows of W2,  tokens]  = W2_e  . act_e^T, epilogue -> y (fp32)
//
// "Swap-AB": the weight matrix is the M operand (128 rows per tile, read from
// HBM exactly once per token tile) and the tokens routed to an expert are the
// N operand (16..256 columns), so a decode step with one token per expert is a
// weight-streaming GEMV on the tensor pipe and a prefill is an ordinary
// grouped GEMM.  Operands are K-major in shared memory, staged by TMA with
// 128-byte swizzle; accumulators live in TMEM (two buffers so the epilogue of
// one tile overlaps the MMAs of the next).
//
// INT8 per-channel weights: a bulk copy brings the int8 tile into a staging
// buffer and four converter warps widen it to f16 (exact for |q| <= 127), either
// into the swizzled shared-memory operand layout or -- decode tiles and the
// 256-token gate/up GEMM (gemm_ts) -- into TMEM, where the MMA reads its A
// operand; the per-row scale is applied to the fp32 accumulator in the epilogue
// (scale is per M row = per TMEM lane).
//
// Warp roles: warp 0 TMA producer, warp 1 TMEM owner and MMA issuer, then the
// epilogue warps (4, or 8 for tiles of 128 columns and more), then the 4 int8
// converter warps (INT8 weights only).
#include "common.cuh"
#include "moe_internal.h"

namespace moe {

struct GemmArgs {
  CUtensorMap a_routed;  // f16 weights [groups * rows_a][K]
  CUtensorMap a_shared;  // f16 shared expert weights [m_limit_shared][K]
  // int8 weights, tile-major (i8_tile_off): a group's matrix a8_group_bytes long,
  // a8_nkb_* 64-column tiles per 128-row tile
  const int8_t* a8_routed;
  const int8_t* a8_shared;
  size_t a8_group_bytes;
  int a8_nkb_routed, a8_nkb_shared;
  CUtensorMap b_routed;  // activations f16 [rows][K]
  CUtensorMap b_shared;
  TileMap map;           // routed / shared unit list (grouped GEMMs)
  int router_grid;       // 1: router mode, units form a plain (m, n, split) grid
  int max_tiles;
  int n_local;           // group id of the shared expert
  int rows_a_routed;     // A rows per routed expert
  int m_limit_routed;    // valid A rows per routed expert
  int m_limit_shared;
  int k_routed, k_shared;
  __half* act_routed;    // gate/up outputs [rows][I]
  __half* act_shared;    // [T][SI]
  int act_ld_routed, act_ld_shared;
  float* y_routed;       // down outputs [rows][H]
  float* y_shared;       // [T][H]
  int y_ld;
  __half* y_half;        // if set: routed down outputs as f16 at row y_row_map[row] (or row)
  const int32_t* y_row_map;
  // router mode (tiles == nullptr: implicit m x n x split grid over implicit_rows tokens)
  int implicit_ntn, implicit_rows, implicit_splits;
  float* logits;         // [split][tokens][logit_ld] partial logit planes
  int logit_ld;
  float logit_scale;
  const float* scale_routed;  // int8 row scales [groups * rows_a]
  const float* scale_shared;  // [m_limit_shared]
  float* kpart;               // split-K partials [tile_id * nsplit + split][128][16] f32
  int* kcount;                // per-tile split arrival counters (zeroed by the tile builder)
  int* err;
};

// Named barrier of the NT epilogue threads (barrier 0 is __syncthreads).
template <int NT>
MOE_DEV void epilogue_bar() { asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory"); }

// TS: the widened f16 A operand lives in TMEM instead of shared memory (INT8
// decode tiles, see gemm_ts).
template <int BN, bool TS = false>
struct TileCfg {
  static constexpr int kStageA = TS ? 0 : kBM * kBK * 2;  // f16 A tile, 16 KiB (none if in TMEM)
  static constexpr int kStageA8 = kBM * kBK;         // int8 staging tile, 8 KiB
  static constexpr int kStageB = BN * kBK * 2;
  // Decode tiles (N <= 64) spread the four K = 16 MMAs of a k-block over four
  // independent TMEM accumulators ("chains"): with a handful of token columns an
  // MMA is short, and MMAs that accumulate into one accumulator wait on each
  // other, so a single chain ran one k-block per ~0.39 us whatever its bytes.  The
  // epilogue adds the chains in a fixed order.  Wide prefill tiles keep one; a
  // 64-column tile with its A operand in TMEM keeps two (room for the A slots).
  static constexpr int kChains = BN <= 32 ? 4 : (BN <= 64 ? (TS ? 2 : 4) : 1);
  static constexpr int kAccCols = kChains * BN;  // one accumulator buffer
  static constexpr int kTmemCols = TS ? 512 : (2 * kAccCols <= 32) ? 32 : (2 * kAccCols <= 64) ? 64
                                   : (2 * kAccCols <= 128) ? 128 : (2 * kAccCols <= 256) ? 256 : 512;
  // accumulator buffers: two (tile i's epilogue overlaps tile i+1's MMAs), one for a
  // 256-column tile with its A operand in TMEM (the A slots take the other half)
  static constexpr int kAccBufs = (TS && BN > 64) ? 1 : 2;
  static constexpr int kAColBase = kAccBufs * kAccCols;  // TS: first column of the A slots
  // Epilogue warps: a 256-column accumulator takes 8 (each TMEM lane quarter
  // twice, splitting the columns) so that draining a tile stays shorter than
  // its MMAs; narrow decode tiles keep 4.
  static constexpr int kEpiWarps = BN >= 128 ? 8 : 4;
};

// Warp roles: 0 TMA producer, 1 TMEM owner + MMA issuer, 2 .. 2+E-1 epilogue,
// then 4 int8 -> f16 converter warps when the weights are INT8.
template <int BN, bool INT8>
__host__ __device__ constexpr int gemm_threads() {
  return 32 * (2 + TileCfg<BN>::kEpiWarps + (INT8 ? 4 : 0));
}

// INT8 decode tiles (N <= 64) widen the int8 weight tile into TMEM (tcgen05.st by
// the converter warps) and the MMA reads its A operand from there: no f16 copy of
// A in shared memory, so a stage is only the int8 tile and the token tile and
// more k-blocks of weights fit in flight per SM; the hand-off to the MMA is a
// TMEM store and a barrier.  128-token tiles keep A in shared memory.
#ifndef MOE_INT8_TMEM_A
#define MOE_INT8_TMEM_A 1
#endif
// 256-token INT8 tiles take the TMEM A path too for the gate/up GEMM
// (MOE_INT8_TMEM_A_PREFILL 1; 2: the down GEMM as well, 0: neither).  The A slots
// then take half of TMEM, so one accumulator buffer and five 40 KiB stages
// instead of two buffers and four 56 KiB stages: gate/up 1.219 -> 1.171 ms at
// 4096 tokens (GLM-4.7 dims), but the down GEMM (24 k-blocks a tile) loses its
// epilogue overlap, 0.676 -> 0.819 ms.
#ifndef MOE_INT8_TMEM_A_PREFILL
#define MOE_INT8_TMEM_A_PREFILL 1
#endif
template <int BN, bool INT8, bool DOWN = false>
__host__ __device__ constexpr bool gemm_ts() {
  return MOE_INT8_TMEM_A && INT8 &&
         (BN <= 64 || (BN == 256 && MOE_INT8_TMEM_A_PREFILL >= (DOWN ? 2 : 1)));
}

// As many stages as fit under the 227 KiB opt-in shared memory per CTA (less the
// alignment slack, barriers and a little static shared memory), up to 8 (12 with
// the A operand in TMEM): the prefill GEMMs are bound by the bytes in flight
// between L2 and the SM (Little's law over the ring), so a fourth INT8 stage at
// BN = 256 pays directly.
constexpr int kGemmBarBytes = 1024;
constexpr int kGemmSmemBudget = 232448 - 1024 - kGemmBarBytes - 512;

#ifndef MOE_GEMM_MAX_STAGES
#define MOE_GEMM_MAX_STAGES 8
#endif
#ifndef MOE_GEMM_MAX_STAGES_TS
#define MOE_GEMM_MAX_STAGES_TS 12
#endif

// k-blocks per pipeline stage.  INT8 decode tiles (N <= 64) widen two 64-column
// k-blocks per stage: each stage costs the converter warps a fixed hand-off
// (wait for the copy, widen, proxy fence, barrier to the MMA thread), and with
// one k-block per stage that cost, not the bytes, set the pace (~0.39 us per
// k-block for 8 KiB of int8, the same as for 16 KiB of f16).  Two k-blocks per
// stage measured 13 % faster at 32 tokens; four (two stages) and a split ring
// (14 single-k-block int8 stages feeding 3 widened slots) measured slower.  f16
// stages and wide prefill tiles keep one k-block.
#ifndef MOE_INT8_DECODE_KPS
#define MOE_INT8_DECODE_KPS 2
#endif
// With the widened A operand in TMEM (gemm_ts) the per-stage cost dominates still
// more: four k-blocks per stage measured 22 % faster than two at 32 tokens (one:
// 20 % slower), whatever the number of TMEM A slots (2 to 14) or accumulator
// chains; a second group of converter warps, and a separate ring for the token
// tiles (so that int8 stages return to the producer once converted) gained nothing.
#ifndef MOE_INT8_DECODE_KPS_TS
#define MOE_INT8_DECODE_KPS_TS 4
#endif

template <int BN, bool INT8, bool DOWN = false>
__host__ __device__ constexpr int gemm_kps() {
  return gemm_ts<BN, INT8, DOWN>() ? (BN <= 64 ? MOE_INT8_DECODE_KPS_TS : 1)
                                   : (INT8 && BN <= 64) ? MOE_INT8_DECODE_KPS : 1;
}

template <int BN, bool INT8, bool DOWN = false>
__host__ __device__ constexpr int gemm_stage_bytes() {
  using C = TileCfg<BN, gemm_ts<BN, INT8, DOWN>()>;
  return gemm_kps<BN, INT8, DOWN>() * (C::kStageA + C::kStageB + (INT8 ? C::kStageA8 : 0));
}

template <int BN, bool INT8, bool DOWN = false>
__host__ __device__ constexpr int gemm_stages() {
  constexpr int s = kGemmSmemBudget / gemm_stage_bytes<BN, INT8, DOWN>();
  constexpr int cap = gemm_ts<BN, INT8, DOWN>() ? MOE_GEMM_MAX_STAGES_TS : MOE_GEMM_MAX_STAGES;
  return s > cap ? cap : s;
}

// TMEM A slots (KPS k-blocks of 32 columns each) in the columns the
// accumulator buffers leave free.
template <int BN, bool INT8, bool DOWN = false>
__host__ __device__ constexpr int gemm_a_slots() {
  using C = TileCfg<BN, gemm_ts<BN, INT8, DOWN>()>;
  return gemm_ts<BN, INT8, DOWN>() ? (C::kTmemCols - C::kAColBase) / (32 * gemm_kps<BN, INT8, DOWN>())
                                   : 0;
}

template <int BN, bool INT8, bool DOWN = false>
__host__ __device__ constexpr size_t gemm_smem_bytes() {
  return 1024 /*align slack*/ +
         static_cast<size_t>(gemm_stages<BN, INT8, DOWN>()) * gemm_stage_bytes<BN, INT8, DOWN>() +
         kGemmBarBytes;
}

// Widen one 128 x 64 int8 tile (as stored: 64-byte rows, 16-byte chunk v of row
// r at chunk v ^ ((r >> 1) & 3), i8_tile_off) to f16 in the 128-byte-swizzled
// K-major layout the MMA descriptor expects (16-byte chunk c of row r lands at
// chunk c ^ (r & 7)).  The stored chunk order makes eight neighbouring rows' reads
// of one chunk hit eight different bank groups.  int8 -> f16 exactly: bias the
// byte to u = q + 128, place it in the mantissa of 1024.0 (0x6400 | u = 1024 + u),
// subtract 1152.
MOE_DEV void convert_row_i8_f16(const int8_t* src_row, uint8_t* dst_tile, int r) {
  const uint4* s4 = reinterpret_cast<const uint4*>(src_row);
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
  const int rot = (r >> 1) & 3;
#pragma unroll
  for (int v = 0; v < 4; ++v) {  // 4 x 16 int8 = 64 elements
    const uint4 q = s4[v ^ rot];
    const uint32_t words[4] = {q.x, q.y, q.z, q.w};
    uint32_t out[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t u = words[i] ^ 0x80808080u;
      uint32_t lo = __byte_perm(u, 0x64646464u, 0x4140);
      uint32_t hi = __byte_perm(u, 0x64646464u, 0x4342);
      __half2 l2 = __hsub2(*reinterpret_cast<__half2*>(&lo), bias);
      __half2 h2 = __hsub2(*reinterpret_cast<__half2*>(&hi), bias);
      out[2 * i] = *reinterpret_cast<uint32_t*>(&l2);
      out[2 * i + 1] = *reinterpret_cast<uint32_t*>(&h2);
    }
    // 16 int8 -> 32 bytes of f16 = chunks 2v and 2v+1 of this row
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int chunk = 2 * v + h;
      uint4* dst = reinterpret_cast<uint4*>(dst_tile + r * 128 + ((chunk ^ (r & 7)) << 4));
      *dst = make_uint4(out[4 * h], out[4 * h + 1], out[4 * h + 2], out[4 * h + 3]);
    }
  }
}

// The same widening into registers for a TMEM A operand, in two steps so that a
// stage's shared-memory reads are all in flight before the first conversion:
// load_row_i8 fetches row r's 64 int8 in k order, widen_i8 turns them into the 32
// columns of one k-block (out[c] holds k = 2c in its lower half and 2c + 1).
MOE_DEV void load_row_i8(const int8_t* src_row, int r, uint4 (&q)[4]) {
  const uint4* s4 = reinterpret_cast<const uint4*>(src_row);
  const int rot = (r >> 1) & 3;
#pragma unroll
  for (int v = 0; v < 4; ++v) q[v] = s4[v ^ rot];
}
MOE_DEV void widen_i8(const uint4 (&q)[4], uint32_t (&out)[32]) {
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    const uint32_t words[4] = {q[v].x, q[v].y, q[v].z, q[v].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t u = words[i] ^ 0x80808080u;
      uint32_t lo = __byte_perm(u, 0x64646464u, 0x4140);
      uint32_t hi = __byte_perm(u, 0x64646464u, 0x4342);
      __half2 l2 = __hsub2(*reinterpret_cast<__half2*>(&lo), bias);
      __half2 h2 = __hsub2(*reinterpret_cast<__half2*>(&hi), bias);
      out[8 * v + 2 * i] = *reinterpret_cast<uint32_t*>(&l2);
      out[8 * v + 2 * i + 1] = *reinterpret_cast<uint32_t*>(&h2);
    }
  }
}

enum GemmMode { MODE_GATEUP = 0, MODE_DOWN = 1, MODE_ROUTER = 2 };

// Unit u of a tile map (see TileMap).  A map that does not describe u (a
// corrupted count) yields a tile that tile_ok rejects.
MOE_DEV Tile tile_at(const TileMap& m, int u, int tot, int splits) {
  Tile t;
  t.group = -1;
  t.m0 = 0;
  t.row0 = 0;
  t.nvalid = 0;
  t.kb0 = t.kb1 = 0;
  t.tile_id = 0;
  t.split = 1 << 16;
  if (splits < 1) return t;
  const int q = u / splits, sidx = u - q * splits;
  int nk;
  if (q < tot) {
    if (m.groups <= 0) return t;
    int lo = 0, hi = m.groups;  // the last group g with pre[g] <= q owns tile q
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (__ldg(m.pre + mid) <= q) lo = mid;
      else hi = mid;
    }
    const int o0 = __ldg(m.off + lo);
    const int cc = __ldg(m.off + lo + 1) - o0;
    const int nt = (cc + m.bn - 1) / m.bn;
    if (nt <= 0) return t;
    const int l = q - __ldg(m.pre + lo);
    const int mm = l / nt, n = l - mm * nt;
    t.group = lo;
    t.m0 = mm * kBM;
    t.row0 = o0 + n * m.bn;
    t.nvalid = min(m.bn, cc - n * m.bn);
    nk = m.nk;
  } else {
    if (m.shared_ntn <= 0) return t;
    const int i = q - tot;
    const int mm = i / m.shared_ntn, n = i - mm * m.shared_ntn;
    t.group = m.shared_group;
    t.m0 = mm * kBM;
    t.row0 = n * m.bn;
    t.nvalid = min(m.bn, m.shared_rows - n * m.bn);
    nk = m.nk_shared;
  }
  t.kb0 = sidx * nk / splits;
  t.kb1 = (sidx + 1) * nk / splits;
  t.split = sidx | (splits << 16);
  t.tile_id = q;
  return t;
}

template <int BN, int MODE, bool INT8>
__global__ void __launch_bounds__(gemm_threads<BN, INT8>(), 1)
    moe_gemm_kernel(const __grid_constant__ GemmArgs args) {
  constexpr bool DOWN = MODE == MODE_DOWN;
  constexpr int STAGES = gemm_stages<BN, INT8, DOWN>();
  constexpr int KPS = gemm_kps<BN, INT8, DOWN>();  // k-blocks per stage
  constexpr bool TS = gemm_ts<BN, INT8, DOWN>();   // widened A operand in TMEM
  using Cfg = TileCfg<BN, TS>;
  constexpr int NA = gemm_a_slots<BN, INT8, DOWN>();  // TMEM A slots (TS)
  constexpr int NCONV = TS ? NA : STAGES;       // "widened" barriers: per A slot or per stage
  // per k-block operand bytes; stage s holds k-blocks [s * KPS, s * KPS + KPS) of each buffer
  constexpr int SA = Cfg::kStageA, SB = Cfg::kStageB, SA8 = Cfg::kStageA8;
  // The MMA runs with N = nvalid rounded up to 16: a partial tile does not pay
  // tensor time for the token columns it does not use.
  constexpr uint32_t TMEM_COLS = Cfg::kTmemCols;
  static_assert(!TS || NA >= 2, "TMEM A ring needs two slots");
  static_assert((2 * STAGES + NCONV + NA + 5) * 8 + 8 <= kGemmBarBytes, "barrier area");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * KPS * SA;
  uint8_t* sA8 = sB + STAGES * KPS * SB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sA8 + (INT8 ? STAGES * KPS * SA8 : 0));
  uint64_t* full = bars;                 // TMA landed (A + B)
  uint64_t* empty = full + STAGES;       // MMA finished reading the stage
  uint64_t* conv = empty + STAGES;       // int8 tile widened to f16 (per stage / A slot)
  uint64_t* aempty = conv + NCONV;       // TS: MMA finished reading an A slot
  uint64_t* tfull = aempty + NA;         // accumulator ready
  uint64_t* tempty = tfull + 2;          // accumulator drained
  uint64_t* mma_done = tempty + 2;       // final drain of in-flight MMAs
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  constexpr int EPI = Cfg::kEpiWarps;
  __shared__ int s_ready[2][EPI];  // epilogue warps' per-tile readiness votes
  __shared__ volatile int s_last; // split-K: this CTA finishes the tile

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Grouped GEMMs read their unit count and K split from the tile map the
  // routing kernels wrote (after pdl_wait below); the router GEMM's units are a
  // plain (m, n, K split) grid derived from the index.
  int map_tot = 0, map_splits = 1, ntiles = 0;
  auto fetch_tile = [&](int ti) {
    if (!args.router_grid) return tile_at(args.map, ti, map_tot, map_splits);
    Tile t;
    const int ntn = args.implicit_ntn, ns = args.implicit_splits;
    const int sidx = ti % ns, mn = ti / ns;
    const int nk = (args.k_routed + kBK - 1) / kBK;
    t.group = 0;
    t.m0 = (mn / ntn) * kBM;
    t.row0 = (mn % ntn) * BN;
    t.nvalid = min(BN, args.implicit_rows - t.row0);
    t.kb0 = sidx * nk / ns;
    t.kb1 = (sidx + 1) * nk / ns;
    t.split = sidx | (ns << 16);
    t.tile_id = mn;
    return t;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int c = 0; c < NCONV; ++c) mbar_init(&conv[c], 4);  // one arrival per converter warp
    for (int a = 0; a < NA; ++a) mbar_init(&aempty[a], 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 32 * EPI);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    if (!INT8) tma_prefetch_desc(&args.a_routed);
    tma_prefetch_desc(&args.b_routed);
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // the prologue above touches only on-chip state; global memory after this
  pdl_wait();
  map_tot = args.router_grid ? 0 : __ldg(args.map.info);
  map_splits = args.router_grid ? 1 : __ldg(args.map.info + 1);
  ntiles = args.router_grid ? args.max_tiles : min(__ldg(args.map.info + 2), args.max_tiles);

  auto tile_ok = [&](const Tile& t) {
    if (t.group < 0 || t.group > args.n_local || t.nvalid <= 0 || t.nvalid > BN) return false;
    const bool sh = t.group == args.n_local;
    const int lim = sh ? args.m_limit_shared : args.m_limit_routed;
    const int nk = ((sh ? args.k_shared : args.k_routed) + kBK - 1) / kBK;
    const int nsplit = t.split >> 16, sidx = t.split & 0xffff;
    if (nsplit < 1 || sidx >= nsplit) return false;
    if (nsplit > 1 && BN != kSplitTileRows && MODE != MODE_ROUTER) return false;
    return t.m0 >= 0 && t.m0 < lim && t.kb0 >= 0 && t.kb0 < t.kb1 && t.kb1 <= nk;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;
      for (int ti = blockIdx.x; ti < ntiles && !*abort_flag; ti += gridDim.x) {
        const Tile t = fetch_tile(ti);
        if (!tile_ok(t)) {
          record_error(args.err, DEV_BAD_TILE);
          continue;
        }
        const bool sh = t.group == args.n_local;
        const CUtensorMap* ma = sh ? &args.a_shared : &args.a_routed;
        const CUtensorMap* mb = sh ? &args.b_shared : &args.b_routed;
        const int arow = sh ? t.m0 : t.group * args.rows_a_routed + t.m0;
        // int8: this row tile's k-blocks are consecutive 8 KiB blocks
        const int8_t* a8 = nullptr;
        if constexpr (INT8) {
          a8 = (sh ? args.a8_shared : args.a8_routed + static_cast<size_t>(t.group) * args.a8_group_bytes) +
               static_cast<size_t>(t.m0 / kBM) * (sh ? args.a8_nkb_shared : args.a8_nkb_routed) * SA8;
        }
        for (int kb = t.kb0; kb < t.kb1; kb += KPS, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          const int n = min(KPS, t.kb1 - kb);  // k-blocks in this stage
          if (!mbar_wait_bounded(&empty[s], ph ^ 1, abort_flag)) {
            *abort_flag = 1;
            record_error(args.err, DEV_TIMEOUT_EMPTY);
            break;
          }
          mbar_arrive_expect_tx(&full[s], n * ((INT8 ? SA8 : SA) + SB));
          // the k-blocks of a tile-major int8 row tile are consecutive: one copy
          if constexpr (INT8) bulk_load(sA8 + s * KPS * SA8, a8 + static_cast<size_t>(kb) * SA8, n * SA8, &full[s]);
          else tma_load_2d(sA + s * SA, ma, kb * kBK, arow, &full[s]);
          for (int j = 0; j < n; ++j)
            tma_load_2d(sB + (s * KPS + j) * SB, mb, (kb + j) * kBK, t.row0, &full[s]);
        }
      }
      // drain: every stage's most recent load must have landed before exit
      for (int j = 0; j < STAGES && j < it; ++j) {
        const int i = it - 1 - j;
        const int s = i % STAGES;
        mbar_wait_drain(&full[s], (i / STAGES) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int it = 0, tl = 0;
      bool issued = false;
      for (int ti = blockIdx.x; ti < ntiles && !*abort_flag; ti += gridDim.x) {
        const Tile t = fetch_tile(ti);
        if (!tile_ok(t)) continue;
        constexpr int NB = Cfg::kAccBufs;
        const int buf = tl % NB;
        if (!mbar_wait_bounded(&tempty[buf], ((tl / NB) & 1) ^ 1, abort_flag)) {
          *abort_flag = 1;
          record_error(args.err, DEV_TIMEOUT_TMEM_EMPTY);
          break;
        }
        tc_fence_after();
        constexpr int CH = Cfg::kChains;
        const uint32_t d = tmem_base + buf * Cfg::kAccCols;
        const uint32_t idesc = idesc_f16_f32(kBM, (t.nvalid + 15) & ~15);
        bool ok = true;
        for (int kb = t.kb0; kb < t.kb1; kb += KPS, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          const int n = min(KPS, t.kb1 - kb);
          const int ca = TS ? it % (NA > 0 ? NA : 1) : s;  // widened barrier / A slot
          const uint32_t cph = TS ? (it / (NA > 0 ? NA : 1)) & 1 : ph;
          if (!mbar_wait_bounded(INT8 ? &conv[ca] : &full[s], cph, abort_flag)) {
            *abort_flag = 1;
            record_error(args.err, DEV_TIMEOUT_FULL);
            ok = false;
            break;
          }
          tc_fence_after();
          for (int j = 0; j < n; ++j) {
            const uint32_t b0 = smem_u32(sB + (s * KPS + j) * SB);
            if constexpr (TS) {
              const uint32_t a0 = tmem_base + Cfg::kAColBase + (ca * KPS + j) * 32;
#pragma unroll
              for (int k = 0; k < kBK / 16; ++k)
                tc_mma_f16_ts(d + (k % CH) * BN, a0 + k * 8, sw128_desc(b0 + k * 32), idesc,
                              (kb + j > t.kb0 || k >= CH) ? 1u : 0u);
            } else {
              const uint32_t a0 = smem_u32(sA + (s * KPS + j) * SA);
#pragma unroll
              for (int k = 0; k < kBK / 16; ++k) {
                // MMA k feeds chain k % CH; a chain's first MMA of the tile starts it
                tc_mma_f16(d + (k % CH) * BN, sw128_desc(a0 + k * 32), sw128_desc(b0 + k * 32), idesc,
                           (kb + j > t.kb0 || k >= CH) ? 1u : 0u);
              }
            }
          }
          tc_commit(&empty[s]);
          if constexpr (TS) tc_commit(&aempty[ca]);
          issued = true;
        }
        if (!ok) break;
        tc_commit(&tfull[buf]);
        ++tl;
      }
      if (issued) {  // make sure no MMA still writes TMEM when it is released
        tc_commit(mma_done);
        mbar_wait_drain(mma_done, 0);
      }
    }
  } else if (warp < 2 + EPI) {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;         // epilogue warp index
    const int q = warp & 3;          // TMEM lane quarter this warp may access
    const int cfirst = (ew >> 2) * 16, cstep = 16 * (EPI / 4);  // its column chunks
    const int r = q * 32 + lane;
    int tl = 0;
    bool range_bad = false;
    for (int ti = blockIdx.x; ti < ntiles; ti += gridDim.x) {
      const Tile t = fetch_tile(ti);
      if (!tile_ok(t)) continue;
      constexpr int NB = Cfg::kAccBufs;
      const int buf = tl % NB;
      // every lane polls; the warp vote re-converges the warp before the
      // .sync.aligned TMEM loads, and the epilogue warps then agree through a
      // double-buffered flag so that all of them take (or skip) the named
      // barriers below together
      const bool my_ready = __all_sync(0xffffffffu, mbar_wait_bounded(&tfull[buf], (tl / NB) & 1, abort_flag));
      if (lane == 0) s_ready[tl & 1][ew] = my_ready ? 1 : 0;
      epilogue_bar<32 * EPI>();
      bool ready = true;
#pragma unroll
      for (int w = 0; w < EPI; ++w) ready = ready && s_ready[tl & 1][w];
      if (!ready) {
        *abort_flag = 1;
        record_error(args.err, DEV_TIMEOUT_TMEM_FULL);
        break;
      }
      tc_fence_after();
      const int nsplit = t.split >> 16;
      const bool sh = t.group == args.n_local;
      const int mrow = t.m0 + r;  // row inside this group's A matrix
      const bool row_ok = mrow < (sh ? args.m_limit_shared : args.m_limit_routed);
      float rs = 1.f;
      if (INT8 && row_ok) {
        rs = sh ? args.scale_shared[mrow]
                : args.scale_routed[static_cast<size_t>(t.group) * args.rows_a_routed + mrow];
      }
      constexpr int CH = Cfg::kChains;
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * Cfg::kAccCols;
      const int ncol = (t.nvalid + 15) & ~15;
      for (int c0 = cfirst; c0 < ncol; c0 += cstep) {
        float v[16];
        tmem_ld16(taddr + c0, v);
#pragma unroll
        for (int ch = 1; ch < CH; ++ch) {  // add the other chains, in chain order
          float w[16];
          tmem_ld16(taddr + ch * BN + c0, w);
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] += w[i];
        }
        if constexpr (BN == kSplitTileRows) {
          if (nsplit > 1) {
            // K split: publish this split's partial, count arrivals; the last
            // split sums all partials in split order and runs the epilogue
            const int sidx = t.split & 0xffff;
            float4* mine = reinterpret_cast<float4*>(
                args.kpart + ((static_cast<size_t>(t.tile_id) * nsplit + sidx) * kBM + r) * 16);
#pragma unroll
            for (int i = 0; i < 4; ++i) mine[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            __threadfence();
            epilogue_bar<32 * EPI>();
            if (threadIdx.x == 64) s_last = (atomicAdd(&args.kcount[t.tile_id], 1) == nsplit - 1) ? 1 : 0;
            epilogue_bar<32 * EPI>();
            if (!s_last) break;  // ncol == 16: this was the only chunk
            __threadfence();
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = 0.f;
            for (int sp = 0; sp < nsplit; ++sp) {
              const float4* pp = reinterpret_cast<const float4*>(
                  args.kpart + ((static_cast<size_t>(t.tile_id) * nsplit + sp) * kBM + r) * 16);
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float4 a = __ldcg(pp + i);
                v[4 * i] += a.x;
                v[4 * i + 1] += a.y;
                v[4 * i + 2] += a.z;
                v[4 * i + 3] += a.w;
              }
            }
          }
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] *= rs;
        if constexpr (MODE == MODE_ROUTER) {
          // router logits: D[router row, token] * 2^-10 -> plane[split][token][row]
          float* plane = args.logits + static_cast<size_t>(t.split & 0xffff) * args.implicit_rows *
                                           args.logit_ld;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int col = c0 + i;
            if (col < t.nvalid && row_ok)
              plane[static_cast<size_t>(t.row0 + col) * args.logit_ld + mrow] = v[i] * args.logit_scale;
          }
        } else if constexpr (!DOWN) {
          // lanes 0-15: gate rows, lanes 16-31: the matching up rows.  Lane l < 16
          // forms the activation of feature l for the even columns, lane l + 16
          // for the odd ones; neighbouring features then pair up across lanes
          // l, l ^ 1 so that every store is a 4-byte half2 (2-byte scattered
          // stores cost the epilogue more than twice the time).
          const int feat = (mrow >> 5) * 16 + (lane & 15);
          __half* dst = sh ? args.act_shared : args.act_routed;
          const int ld = sh ? args.act_ld_shared : args.act_ld_routed;
          float a[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float o = __shfl_xor_sync(0xffffffffu, (lane < 16) ? v[2 * j + 1] : v[2 * j], 16);
            const float g = (lane < 16) ? v[2 * j] : o;
            const float u = (lane < 16) ? o : v[2 * j + 1];
            a[j] = silu_f(g) * u;
          }
#pragma unroll
          for (int j = 0; j < 8; j += 2) {
            const float o = __shfl_xor_sync(0xffffffffu, (lane & 1) ? a[j] : a[j + 1], 1);
            const float lo = (lane & 1) ? o : a[j];
            const float hi = (lane & 1) ? a[j + 1] : o;
            const int col = c0 + 2 * (j + (lane & 1)) + (lane >> 4);
            if (col < t.nvalid && row_ok) {
              range_bad |= !fits_f16(lo) || !fits_f16(hi);
              *reinterpret_cast<__half2*>(dst + static_cast<size_t>(t.row0 + col) * ld + (feat & ~1)) =
                  __floats2half2_rn(lo, hi);
            }
          }
        } else {
          if (!sh && args.y_half) {
            // features mrow & ~1 and | 1 pair up across lanes l, l ^ 1: even lanes
            // store column i, odd lanes column i + 1, each as one half2
#pragma unroll
            for (int i = 0; i < 16; i += 2) {
              const float o = __shfl_xor_sync(0xffffffffu, (lane & 1) ? v[i] : v[i + 1], 1);
              const float lo = (lane & 1) ? o : v[i];
              const float hi = (lane & 1) ? v[i + 1] : o;
              const int col = c0 + i + (lane & 1);
              if (col < t.nvalid && row_ok) {
                range_bad |= !fits_f16(lo) || !fits_f16(hi);
                const int orow = args.y_row_map ? args.y_row_map[t.row0 + col] : t.row0 + col;
                *reinterpret_cast<__half2*>(args.y_half + static_cast<size_t>(orow) * args.y_ld + (mrow & ~1)) =
                    __floats2half2_rn(lo, hi);
              }
            }
          } else {
            float* dst = sh ? args.y_shared : args.y_routed;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int col = c0 + i;
              if (col < t.nvalid && row_ok) dst[static_cast<size_t>(t.row0 + col) * args.y_ld + mrow] = v[i];
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
      ++tl;
    }
    // an f16 activation / expert output that overflowed is reported, not passed on
    // silently as inf (moe_status -> MOE_ERR_RANGE)
    if (__any_sync(0xffffffffu, range_bad) && lane == 0) record_error(args.err, DEV_RANGE);
  } else if constexpr (INT8) {
    // ------------------------------------------------------------ int8 -> f16
    // one A row per thread; with A in TMEM a warp may only write its own quarter
    // of the TMEM lanes (warp % 4), so its rows follow that quarter
    const int r = TS ? (warp & 3) * 32 + lane : (warp - 2 - EPI) * 32 + lane;
    int it = 0;
    for (int ti = blockIdx.x; ti < ntiles && !*abort_flag; ti += gridDim.x) {
      const Tile t = fetch_tile(ti);
      if (!tile_ok(t)) continue;
      bool ok = true;
      for (int kb = t.kb0; kb < t.kb1; kb += KPS, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        const int n = min(KPS, t.kb1 - kb);
        if constexpr (TS) {
          const int a = it % NA;
          // the A slot must be free (the MMAs of its previous use completed) and
          // the int8 tile in place
          if (!__all_sync(0xffffffffu, mbar_wait_bounded(&aempty[a], ((it / NA) & 1) ^ 1, abort_flag)) ||
              !__all_sync(0xffffffffu, mbar_wait_bounded(&full[s], ph, abort_flag))) {
            *abort_flag = 1;
            record_error(args.err, DEV_TIMEOUT_CONV);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t ta = tmem_base + (static_cast<uint32_t>((warp & 3) * 32) << 16) +
                              Cfg::kAColBase + a * KPS * 32;
          uint4 q[KPS][4];
#pragma unroll
          for (int j = 0; j < KPS; ++j)
            if (j < n) load_row_i8(reinterpret_cast<const int8_t*>(sA8 + (s * KPS + j) * SA8 + r * kBK), r, q[j]);
#pragma unroll
          for (int j = 0; j < KPS; ++j)
            if (j < n) {
              uint32_t w[32];
              widen_i8(q[j], w);
              tmem_st32_nowait(ta + j * 32, w);
            }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&conv[a]);
          continue;
        }
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[s], ph, abort_flag))) {
          *abort_flag = 1;
          record_error(args.err, DEV_TIMEOUT_CONV);
          ok = false;
          break;
        }
        for (int j = 0; j < n; ++j)
          convert_row_i8_f16(reinterpret_cast<const int8_t*>(sA8 + (s * KPS + j) * SA8 + r * kBK),
                             sA + (s * KPS + j) * SA, r);
        // each thread makes its rows visible to the tensor core's (async) proxy; the
        // warp then arrives once: 4 arrivals per stage instead of 128 serialised ones
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[s]);
      }
      if (!ok) break;
    }
  }

  // the next kernel may launch now (released after the tile loop rather than at
  // entry, so that its waiting CTAs never sit beside this kernel's tiles; the two
  // placements measured the same)
  pdl_release();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ launcher
template <int BN, int MODE, bool INT8>
static cudaError_t run_gemm(const GemmArgs& a, int grid, cudaStream_t s) {
  constexpr size_t smem = gemm_smem_bytes<BN, INT8, MODE == MODE_DOWN>();
  static bool attr_set[64] = {};  // per instantiation and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t st = cudaFuncSetAttribute(moe_gemm_kernel<BN, MODE, INT8>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(smem));
    if (st != cudaSuccess) return st;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  return pdl_launch(moe_gemm_kernel<BN, MODE, INT8>, dim3(grid), dim3(gemm_threads<BN, INT8>()),
                    smem, s, a);
}

template <bool DOWN, bool INT8>
static cudaError_t dispatch_bn(const GemmArgs& a, int bn, int grid, cudaStream_t s) {
  constexpr int M = DOWN ? MODE_DOWN : MODE_GATEUP;
  switch (bn) {
    case 16: return run_gemm<16, M, INT8>(a, grid, s);
    case 32: return run_gemm<32, M, INT8>(a, grid, s);
    case 64: return run_gemm<64, M, INT8>(a, grid, s);
    case 128: return run_gemm<128, M, INT8>(a, grid, s);
    case 192:  // 16-bit prefill tiles of experts with few tokens (prefill_bn)
      if constexpr (!INT8) return run_gemm<192, M, INT8>(a, grid, s);
      return cudaErrorInvalidValue;
    case 256: return run_gemm<256, M, INT8>(a, grid, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_gemm(const Plan& p, const WsLayout& L, char* ws, bool down, int T,
                        cudaStream_t s) {
  return launch_gemm(p, L, ws, down, GemmIO{T * p.K, T, nullptr, nullptr, p.n_local}, s);
}

cudaError_t launch_gemm(const Plan& p, const WsLayout& L, char* ws, bool down, const GemmIO& io,
                        cudaStream_t s) {
  GemmArgs a{};
  std::string err;
  const int rows = io.routed_rows;
  const int T = io.shared_rows;
  const int bn = L.bn;
  const bool has_sh = p.SI > 0;
  __half* h16 = reinterpret_cast<__half*>(ws + L.h16);
  __half* xg = reinterpret_cast<__half*>(ws + L.xg);
  __half* act = reinterpret_cast<__half*>(ws + L.act);
  __half* act_s = reinterpret_cast<__half*>(ws + L.act_s);
  if (!down) {
    a.a_routed = p.tm_w13;
    a.a_shared = has_sh ? p.tm_ws13 : p.tm_w13;
    if (!make_tmap_2d(&a.b_routed, xg, false, p.H, rows, kBK, bn, true, &err) ||
        !make_tmap_2d(&a.b_shared, h16, false, p.H, T, kBK, bn, true, &err)) {
      set_error(err);
      return cudaErrorInvalidValue;
    }
    a.rows_a_routed = 2 * p.I;
    a.m_limit_routed = 2 * p.I;
    a.m_limit_shared = 2 * p.SI;
    a.k_routed = p.H;
    a.k_shared = p.H;
    a.scale_routed = p.w.s13;
    a.scale_shared = p.w.ss13;
    if (p.int8) {
      a.a8_routed = static_cast<const int8_t*>(p.w.w13);
      a.a8_shared = has_sh ? static_cast<const int8_t*>(p.w.ws13) : a.a8_routed;
      a.a8_group_bytes = i8_pad_rows(2 * p.I) * i8_pad_cols(p.H);
      a.a8_nkb_routed = a.a8_nkb_shared = static_cast<int>(i8_pad_cols(p.H) / kBK);
    }
  } else {
    a.a_routed = p.tm_w2;
    a.a_shared = has_sh ? p.tm_ws2 : p.tm_w2;
    if (!make_tmap_2d(&a.b_routed, act, false, p.I, rows, kBK, bn, true, &err) ||
        !make_tmap_2d(&a.b_shared, has_sh ? act_s : act, false, has_sh ? p.SI : p.I,
                      has_sh ? T : rows, kBK, bn, true, &err)) {
      set_error(err);
      return cudaErrorInvalidValue;
    }
    a.rows_a_routed = p.H;
    a.m_limit_routed = p.H;
    a.m_limit_shared = p.H;
    a.k_routed = p.I;
    a.k_shared = has_sh ? p.SI : p.I;
    a.scale_routed = p.w.s2;
    a.scale_shared = p.w.ss2;
    if (p.int8) {
      a.a8_routed = static_cast<const int8_t*>(p.w.w2);
      a.a8_shared = has_sh ? static_cast<const int8_t*>(p.w.ws2) : a.a8_routed;
      a.a8_group_bytes = i8_pad_rows(p.H) * i8_pad_cols(p.I);
      a.a8_nkb_routed = static_cast<int>(i8_pad_cols(p.I) / kBK);
      a.a8_nkb_shared = static_cast<int>(i8_pad_cols(has_sh ? p.SI : p.I) / kBK);
    }
  }
  const int32_t* pre = reinterpret_cast<const int32_t*>(ws + L.tile_pre);
  a.map.pre = down ? pre + (io.groups + 1) : pre;
  a.map.off = reinterpret_cast<const int32_t*>(ws + L.offsets);
  a.map.info = reinterpret_cast<const int32_t*>(ws + L.tile_info) + (down ? 4 : 0);
  a.map.groups = io.groups;
  a.map.bn = bn;
  a.map.mt = (a.m_limit_routed + kBM - 1) / kBM;
  a.map.mt_shared = (a.m_limit_shared + kBM - 1) / kBM;
  a.map.shared_ntn = (has_sh && T > 0) ? (T + bn - 1) / bn : 0;
  a.map.shared_rows = T;
  a.map.shared_group = p.n_local;
  a.map.nk = (a.k_routed + kBK - 1) / kBK;
  a.map.nk_shared = (a.k_shared + kBK - 1) / kBK;
  a.router_grid = 0;
  a.n_local = p.n_local;
  a.act_routed = act;
  a.act_shared = act_s;
  a.act_ld_routed = p.I;
  a.act_ld_shared = p.SI;
  a.y_routed = reinterpret_cast<float*>(ws + L.y);
  a.y_shared = reinterpret_cast<float*>(ws + L.y_s);
  a.y_ld = p.H;
  a.y_half = io.y_half;
  a.y_row_map = io.y_row_map;
  a.kpart = reinterpret_cast<float*>(ws + L.kpart);
  a.kcount = reinterpret_cast<int*>(ws + (down ? L.kcount2 : L.kcount1));
  a.err = p.d_err;
  const int max_units = (down ? L.max_tiles2 : L.max_tiles1) * kMaxKSplit;
  a.max_tiles = max_units;
  // persistent: one CTA per SM (extra CTAs exit at once when the list is short)
  const int grid = max_units < p.num_sms ? max_units : p.num_sms;
  if (grid <= 0) return cudaSuccess;
  if (p.int8) return down ? dispatch_bn<true, true>(a, bn, grid, s) : dispatch_bn<false, true>(a, bn, grid, s);
  return down ? dispatch_bn<true, false>(a, bn, grid, s) : dispatch_bn<false, false>(a, bn, grid, s);
}

// Router logits on the tensor cores for prefill batches: D = A . B^T with
// A = f16(W * 2^10) (router rows, bind time) and B = h16 (the normalised f16
// token rows that dispatch gathers), K = H split into `splits` ranges whose
// fp32 partial logits land in separate planes; the selection kernel adds the
// planes in split order.  These logits carry f16 operand error (~2e-3 absolute
// at most for GLM-4.7 shapes): they only pick candidates, and the selection
// kernel recomputes the chosen logits in fp32.
int router_tc_splits(const Plan& p, int T) {
  const int units = ((p.router_rows + kBM - 1) / kBM) * ((T + 255) / 256);
  const int nk = (p.H + kBK - 1) / kBK;
  int best = 1;
  double best_eff = 0.0;
  for (int s = 1; s <= kRouterMaxSplit && nk / s >= 8; ++s) {
    const int u = units * s;
    const int rounds = (u + p.num_sms - 1) / p.num_sms;
    const double eff = static_cast<double>(u) / (static_cast<double>(rounds) * p.num_sms);
    if (eff > best_eff + 0.02) {
      best_eff = eff;
      best = s;
    }
  }
  return best;
}

cudaError_t launch_router_gemm(const Plan& p, const WsLayout& L, char* ws, int T, cudaStream_t s) {
  constexpr int BN = 256;
  GemmArgs a{};
  std::string err;
  a.a_routed = p.tm_rw16;
  a.a_shared = p.tm_rw16;
  if (!make_tmap_2d(&a.b_routed, ws + L.h16, false, p.H, T, kBK, BN, true, &err)) {
    set_error(err);
    return cudaErrorInvalidValue;
  }
  a.b_shared = a.b_routed;
  a.router_grid = 1;
  const int mt = (p.router_rows + kBM - 1) / kBM;
  a.implicit_ntn = (T + BN - 1) / BN;
  a.implicit_rows = T;
  a.implicit_splits = router_tc_splits(p, T);
  a.max_tiles = mt * a.implicit_ntn * a.implicit_splits;
  a.n_local = 1;  // no shared group in this launch
  a.rows_a_routed = 0;
  a.m_limit_routed = p.router_rows;
  a.m_limit_shared = p.router_rows;
  a.k_routed = p.H;
  a.k_shared = p.H;
  a.logits = reinterpret_cast<float*>(ws + L.logits);
  a.logit_ld = p.router_rows;
  a.logit_scale = 1.0f / kRouterWeightScale;
  a.err = p.d_err;
  const int grid = a.max_tiles < p.num_sms ? a.max_tiles : p.num_sms;
  return run_gemm<BN, MODE_ROUTER, false>(a, grid, s);
}

// A plain f16 GEMM on the same kernel (router-grid mode): planes[s][t][r] = the
// K-split s partial of sum_k A[r][k] * B[t][k], A = `a_map` (m_rows x K, f16,
// 64 x 128 boxes), B = b (T x K f16, row-major).  The caller adds the planes in
// split order (the attention projections fold that sum into their next kernel).
// The split count minimises a simple time model: the larger of the tensor work
// (~1.25 PFLOP/s) and the weight stream (~6.5 TB/s), divided by the fraction of
// SM-rounds the tiles fill, plus each extra plane written and read back once.
int dense_gemm_splits(int m_rows, int T, int K, int num_sms) {
  const int units = ((m_rows + kBM - 1) / kBM) * ((T + 255) / 256);
  const int nk = (K + kBK - 1) / kBK;
  const double flops_s = 2.0 * m_rows * T * K / 1.25e15;
  const double weights_s = 2.0 * m_rows * K / 6.5e12;
  const double plane_s = 8.0 * m_rows * T / 6.5e12;
  int best = 1;
  double best_s = 0.0;
  for (int sp = 1; sp <= kRouterMaxSplit && nk / sp >= 8; ++sp) {
    const int u = units * sp;
    const int rounds = (u + num_sms - 1) / num_sms;
    const double eff = static_cast<double>(u) / (static_cast<double>(rounds) * num_sms);
    const double t_s = std::max(flops_s, weights_s) / eff + (sp - 1) * plane_s;
    if (sp == 1 || t_s < 0.98 * best_s) {
      best_s = t_s;
      best = sp;
    }
  }
  return best;
}

cudaError_t launch_dense_gemm(const CUtensorMap& a_map, int m_rows, int K, const __half* b, int T,
                              float* planes, int splits, int* err, int num_sms, cudaStream_t s) {
  constexpr int BN = 256;
  GemmArgs a{};
  std::string emsg;
  a.a_routed = a_map;
  a.a_shared = a_map;
  if (!make_tmap_2d(&a.b_routed, b, false, K, T, kBK, BN, true, &emsg)) {
    set_error(emsg);
    return cudaErrorInvalidValue;
  }
  a.b_shared = a.b_routed;
  a.router_grid = 1;
  const int mt = (m_rows + kBM - 1) / kBM;
  a.implicit_ntn = (T + BN - 1) / BN;
  a.implicit_rows = T;
  a.implicit_splits = splits;
  a.max_tiles = mt * a.implicit_ntn * splits;
  a.n_local = 1;
  a.rows_a_routed = 0;
  a.m_limit_routed = m_rows;
  a.m_limit_shared = m_rows;
  a.k_routed = K;
  a.k_shared = K;
  a.logits = planes;
  a.logit_ld = m_rows;
  a.logit_scale = 1.0f;
  a.err = err;
  const int grid = a.max_tiles < num_sms ? a.max_tiles : num_sms;
  return run_gemm<BN, MODE_ROUTER, false>(a, grid, s);
}

}  // namespace moe
