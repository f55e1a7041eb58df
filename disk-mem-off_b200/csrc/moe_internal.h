// Internal plan / workspace structures shared by the .cu files of libmoe_sm100.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "../../include/moe_sm100.h"

namespace moe {

// Launches a forward kernel chained to the previous kernel of the stream
// (programmatic stream serialisation; the kernel calls pdl_enter / pdl_wait
// before it touches global memory).
template <typename... KArgs, typename... Args>
inline cudaError_t pdl_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Statement form of pdl_launch for launchers that return cudaError_t.
#define MOE_PDL(...)                                  \
  do {                                                \
    const cudaError_t pdl_st_ = pdl_launch(__VA_ARGS__); \
    if (pdl_st_ != cudaSuccess) return pdl_st_;       \
  } while (0)

constexpr int kBM = 128;          // GEMM tile rows (weight rows, swap-AB)
constexpr int kBK = 64;           // GEMM k-block (one 128-byte swizzle atom of f16)
constexpr int kPermChunk = 1024;  // tokens per permutation chunk (bitmask width)
constexpr int kMaxTopK = 32;
// Router weights are scaled by 2^10 before their f16 copy for the prefill
// tensor-core router, so that ~1e-2 weights keep full f16 precision.
constexpr float kRouterWeightScale = 1024.0f;
// The prefill router GEMM splits K into at most this many partial logit planes.
constexpr int kRouterMaxSplit = 4;
// Prefill routing keeps the K + kRefineMargin best tensor-core candidates of a
// token (kCandMax slots) for the fp32 re-decision.
constexpr int kRefineMargin = 12;
constexpr int kCandMax = kMaxTopK + kRefineMargin;

// One unit of work for the grouped GEMM: weight rows [m0, m0+128) of group
// `group` (local routed expert index, or n_local for the shared expert)
// against activation rows [row0, row0 + nvalid) of that group's B matrix, over
// k-blocks [kb0, kb1).  A tile whose K is split across `nsplit` units carries
// its split index and a tile id; the unit that finishes last sums the splits.
struct Tile {
  int group;
  int m0;
  int row0;
  int nvalid;
  int kb0, kb1;
  int split;   // split index | (nsplit << 16)
  int tile_id;
};

// The unit list of one grouped-GEMM launch, in device memory, written by the
// routing kernels: routed tiles are numbered expert-major (group g owns tiles
// [pre[g], pre[g+1]), weight m-tile outer, token tile inner), the shared
// expert's tiles follow, and each tile expands into `splits` adjacent K-split
// units.  The GEMM derives unit u's Tile from this map (tile_at), so routing
// writes E+1 prefix entries per launch instead of a list of every unit.
struct TileMap {
  const int32_t* pre;   // [groups + 1] routed tile prefix; pre[groups] = routed tiles
  const int32_t* off;   // [groups + 1] first row of each group in the B operand
  const int32_t* info;  // [3]: routed tiles, K splits, units
  int groups;           // routed groups (experts of this launch)
  int bn;               // token rows per tile
  int mt;               // weight m-tiles per routed group
  int mt_shared, shared_ntn, shared_rows, shared_group;
  int nk, nk_shared;    // k-blocks of routed / shared tiles
};

constexpr int kMaxKSplit = 4;       // K splits per tile for small decode batches
constexpr int kSplitTileRows = 16;  // split-K only with 16-token tiles (BN = 16)

// INT8 weights are stored tile-major: each 128-row x 64-column tile of a matrix
// is one contiguous 8 KiB block (its rows 64 bytes apart), tiles ordered by row
// tile, then column tile; rows are padded to 128 and columns to 64 with zeros.
// Inside a row the four 16-byte chunks are permuted, chunk c at c ^ ((row >> 1) & 3),
// so that the GEMM's converter threads (one row each, reading chunk c together)
// meet no shared-memory bank conflicts.  One bulk copy fetches a whole k-block of
// weights as a single contiguous transfer.
constexpr int kI8TileRows = 128, kI8TileCols = 64;
static_assert(kI8TileRows == kBM && kI8TileCols == kBK, "an int8 tile is one GEMM k-block of A");
__host__ __device__ inline size_t i8_pad_rows(int m) {
  return (static_cast<size_t>(m) + kI8TileRows - 1) / kI8TileRows * kI8TileRows;
}
__host__ __device__ inline size_t i8_pad_cols(int k) {
  return (static_cast<size_t>(k) + kI8TileCols - 1) / kI8TileCols * kI8TileCols;
}
// byte offset of element (row, col) in a tile-major matrix of kpad padded columns
__host__ __device__ inline size_t i8_tile_off(int row, int col, size_t kpad) {
  const int rr = row % kI8TileRows, cc = col % kI8TileCols;
  const int chunk = (cc >> 4) ^ ((rr >> 1) & 3);
  return static_cast<size_t>(row / kI8TileRows) * kI8TileRows * kpad +
         static_cast<size_t>(col / kI8TileCols) * (kI8TileRows * kI8TileCols) +
         static_cast<size_t>(rr) * kI8TileCols + (chunk << 4) + (cc & 15);
}

struct DeviceWeights {
  // Packed, HBM-resident weights.  W13 rows are interleaved in groups of 32:
  // 16 gate_proj rows then the 16 matching up_proj rows, so one TMEM lane
  // quarter holds both halves of 16 SwiGLU features.  f16 matrices are
  // row-major; int8 ones tile-major (above), each expert padded on its own.
  void* w13 = nullptr;   // f16 or int8 [E_local][2I][H]
  void* w2 = nullptr;    // f16 or int8 [E_local][H][I]
  void* ws13 = nullptr;  // shared expert [2SI][H]
  void* ws2 = nullptr;   // shared expert [H][SI]
  float* s13 = nullptr;  // int8 row scales [E_local][2I] (packed-row order)
  float* s2 = nullptr;   // [E_local][H]
  float* ss13 = nullptr; // [2SI]
  float* ss2 = nullptr;  // [H]
  float* norm_w = nullptr;    // [H]
  float* router_w = nullptr;  // [E (+1 shared gate row)][H]
  float* bias = nullptr;      // [E] or null
  __half* rw16 = nullptr;     // [E (+1)][H] f16(W * 2^10) (prefill tensor-core router)
};

struct Plan {
  MoeConfig cfg{};
  int device = 0;
  int num_sms = 148;
  int E = 0, K = 0, H = 0, I = 0, SI = 0;
  int e_begin = 0, e_end = 0, n_local = 0;
  int router_rows = 0;
  bool int8 = false;
  bool bound = false;
  DeviceWeights w;
  void* weights_alloc = nullptr;
  size_t weights_bytes = 0;
  int* d_err = nullptr;        // device error word
  CUtensorMap tm_w13{}, tm_w2{}, tm_ws13{}, tm_ws2{};
  CUtensorMap tm_rw16{};
  bool router_tc = false;      // tensor-core router available for prefill batches
};

// Workspace carve-up for one forward of T tokens (offsets in bytes).
struct WsLayout {
  size_t h16, xg, act, act_s, y, y_s, logits, part, ss_part, rms, counters, ids, wts, sgate;
  size_t cand, ncand, exact;  // prefill router: candidate ids, rows to recompute, fp32 logits
  size_t bm, hist, base, offsets, perm, slot_row;
  size_t tile_pre;   // [2][groups + 1] routed tile prefix per GEMM (gate/up, down)
  size_t tile_info;  // [2][4]: routed tiles, K splits, units per GEMM
  size_t kpart, kcount1, kcount2;  // split-K partials [units][128][16] f32, per-tile counters
  int max_split_tiles;             // tiles a launch may split (0 = never)
  size_t total;
  int nchunks, max_tiles1, max_tiles2, bn;
};

WsLayout ws_layout(const Plan& p, int T);
WsLayout ws_layout_ep_experts(const Plan& p, int R, int expect);
WsLayout ws_layout_ep_gathered(const Plan& p, int rows, int cap);

// Router launch geometry: rx router-row tiles x splits K-splits x tz token tiles.
struct RouterGeom {
  int rx, tz, splits, k_per_split;
};
RouterGeom router_geometry(const Plan& p, int T);

constexpr int kTailMaxT = 256;  // decode: one CTA does top-k + permutation + tile lists
bool route_uses_tail(const Plan& p, int T);
bool route_uses_small(const Plan& p, int T);  // one-launch routing of small decode batches

// ------------------------------------------------------------ launchers
// Router (+ RMSNorm), top-k, permutation and tile lists; with `dispatch` also
// the normalised f16 rows of every routed slot (xg) and of the shared expert (h16).
cudaError_t launch_route(const Plan& p, const WsLayout& L, char* ws, const float* x, int T,
                         bool dispatch, cudaStream_t s, __half* xg_out = nullptr);
// Where the expert keys of received rows sit: row t has per_row slots whose keys
// are keys[t * key_ld + k] - key_base (k < per_row); pad_mode as perm_hist_kernel
// (0 every key must be a resident expert, 1 negative keys are unused rows,
// 2 keys outside the resident range are skipped).
struct RowKeys {
  const int32_t* keys;
  int key_ld;
  int per_row;
  int key_base;
  int pad_mode;
};
// Expert-parallel helpers: group the slots of `n` received rows by their local
// expert key (stable: receive order inside an expert), gather the rows of the
// kept slots into L.xg and build the tile lists; and the tile lists of the shared
// expert alone for T local tokens.
cudaError_t launch_group_rows(const Plan& p, const WsLayout& L, char* ws, const RowKeys& k,
                              const __half* rows, int row_ld, int n, cudaStream_t s);
// Fixed-capacity send rows of the expert-parallel exchange (after launch_route
// without dispatch): [world * cap] rows of H + 8 f16, tails carrying local ids.
cudaError_t launch_ep_pack(const Plan& p, const WsLayout& L, char* ws, const float* x, int T,
                           int cap, __half* send, cudaStream_t s);
// Token-replicated exchange.  Row width in f16 elements of one token record:
// H normalised values, then K int32 global expert ids and K fp32 weights,
// padded to 16 bytes.
int ep_token_row_halves(const Plan& p);
// [cap] token records of the local T tokens (after launch_route without
// dispatch); rows T..cap-1 carry expert id -1 in every slot.  Also h16 for the
// shared expert.
cudaError_t launch_ep_token_pack(const Plan& p, const WsLayout& L, char* ws, const float* x, int T,
                                 int cap, __half* send, cudaStream_t s);
// partial[t] = sum over the slots k of token record t whose expert is resident
// of w_k * y[slot_row[t*K + k]] (fp32, slot order), zero for a token without one.
cudaError_t launch_ep_partial(const Plan& p, const __half* rows, int n, const __half* y,
                              const int32_t* slot_row, float* partial, cudaStream_t s);
// Token-replicated exchange over peer memory (p2p.cu): every rank's buffers as
// mapped in this process, rank d at index d (d == rank: this rank's own).
constexpr int kMaxP2PRanks = 8;
struct P2PPeers {
  void* recv[kMaxP2PRanks];   // [world*cap][ep_token_row_halves] f16 token records
  float* part[kMaxP2PRanks];  // [world][cap][H] fp32 partial sums
  int* flags[kMaxP2PRanks];   // [2][world] int32 epochs: records, partials
};
cudaError_t launch_p2p_pack(const Plan& p, const WsLayout& L, char* ws, const float* x, int T,
                            int cap, int rank, int world, const P2PPeers& peers, int epoch,
                            int* done, cudaStream_t s);
cudaError_t launch_p2p_wait(const int* flags, int world, int epoch, long long limit, int* err,
                            cudaStream_t s);
cudaError_t launch_p2p_partial(const Plan& p, const __half* rows, int cap, const __half* y,
                               const int32_t* slot_row, int rank, int world, const P2PPeers& peers,
                               int epoch, int* done, cudaStream_t s);
cudaError_t launch_p2p_combine(const Plan& p, const float* x, const float* part, int cap, int world,
                               const float* y_s, const float* sgate, float* out, int T,
                               cudaStream_t s);
// out = x + (partial + shared expert), the combine of the token-replicated exchange.
cudaError_t launch_combine_partial(const Plan& p, const float* x, const float* partial,
                                   const float* y_s, const float* sgate, float* out, int T,
                                   cudaStream_t s);
cudaError_t launch_shared_tiles(const Plan& p, const WsLayout& L, char* ws, int T, cudaStream_t s);
cudaError_t launch_row_prep(const Plan& p, const WsLayout& L, char* ws, const float* x, int T,
                            cudaStream_t s);
cudaError_t launch_router_gemm(const Plan& p, const WsLayout& L, char* ws, int T, cudaStream_t s);
bool route_uses_tc_router(const Plan& p, int T);
int router_tc_splits(const Plan& p, int T);
// Plain f16 GEMM with fp32 K-split planes (attention projections); see gemm_tc.cu.
int dense_gemm_splits(int m_rows, int T, int K, int num_sms);
cudaError_t launch_dense_gemm(const CUtensorMap& a_map, int m_rows, int K, const __half* b, int T,
                              float* planes, int splits, int* err, int num_sms, cudaStream_t s);
// rms[t] = sqrt(mean(x_t^2) + eps), h16[t] = f16(w * (x_t / rms[t])) for T rows.
cudaError_t launch_norm_rows(const float* x, const float* w, int H, float eps, int T, float* rms,
                             __half* h16, int* err, cudaStream_t s);
// Token rows are read as float4 vectors and by bulk copies.
inline bool misaligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) != 0; }
cudaError_t launch_scale_router_weights(const float* w, __half* rw16, int rows, int H, int* err,
                                        cudaStream_t s);
cudaError_t launch_gemm(const Plan& p, const WsLayout& L, char* ws, bool down, int T,
                        cudaStream_t s);
// Rows of the routed / shared B operands and an optional f16 routed output
// (expert-parallel path: written straight into receive order through y_row_map).
struct GemmIO {
  int routed_rows;
  int shared_rows;
  __half* y_half;
  const int32_t* y_row_map;
  int groups;  // routed groups whose tile map the routing kernels wrote
};
cudaError_t launch_gemm(const Plan& p, const WsLayout& L, char* ws, bool down, const GemmIO& io,
                        cudaStream_t s);

cudaError_t launch_combine_half(const Plan& p, const float* x, const __half* y, const float* y_s,
                                const int32_t* slot_row, const float* wts, const float* sgate,
                                float* out, int T, cudaStream_t s);
cudaError_t launch_ep_meta(const Plan& p, const int32_t* perm, const int32_t* ids,
                           const int32_t* offsets, int n, int32_t* send_experts,
                           int32_t* send_offsets, cudaStream_t s);

// weight packing (bind)
cudaError_t launch_pack_rows(const void* src, int src_dtype, void* dst, bool to_int8,
                             float* dst_scale, int rows, int cols, int* range_err,
                             cudaStream_t s);
cudaError_t launch_pack_w13(const void* gate, const void* up, int src_dtype, void* dst,
                            bool to_int8, float* dst_scale, int inter, int cols,
                            int* range_err, cudaStream_t s);
cudaError_t launch_copy_i8_w13(const int8_t* gate, const int8_t* up, const __half* gs,
                               const __half* us, int8_t* dst, float* dst_scale, int inter,
                               int cols, cudaStream_t s);
cudaError_t launch_copy_i8_rows(const int8_t* src, const __half* ss, int8_t* dst,
                                float* dst_scale, int rows, int cols, cudaStream_t s);
cudaError_t launch_to_f32(const void* src, int src_dtype, float* dst, int64_t n,
                          cudaStream_t s);

// source dtypes understood by the packers
enum SrcDtype { SRC_F32 = 0, SRC_F16 = 1, SRC_BF16 = 2, SRC_I8 = 3 };

// tensor maps
bool make_tmap_2d(CUtensorMap* map, const void* base, bool int8, uint64_t inner, uint64_t rows,
                  uint32_t box_inner, uint32_t box_rows, bool swizzle128, std::string* err);

void set_error(const std::string& msg);

}  // namespace moe

// The opaque handle of the C ABI wraps one plan.
struct MoePlan {
  moe::Plan p;
};
