/*
 * libmoe_sm100 -- C ABI of the B200 (sm_100a) MoE feed-forward block.
 *
 * Drop-in device path for the sparse expert layer of disk-mem-off's NumPy
 * executors.  Plain pointers, sizes and int status codes only: every entry
 * point returns MOE_OK (0) or an MOE_ERR_* code and never aborts; the text of
 * the last error of the calling thread is available from moe_last_error().
 * Device pointers are CUDA global-memory addresses; `stream` is a
 * cudaStream_t (NULL = legacy default stream).  All compute calls are
 * stream-ordered and asynchronous.
 *
 * Reference interfaces replaced (paths inside the disk-mem-off project):
 *   moe_forward      -> GLM4MoeExecutor._moe_mlp_block
 *                       offload_runtime/executors/glm4_moe.py:176-240, and
 *                       Qwen3NextExecutor._moe_mlp_block
 *                       offload_runtime/executors/qwen3_next.py:273-333
 *   moe_route        -> the router / top-k / dispatch part of the same functions
 *                       (glm4_moe.py:177-215, qwen3_next.py:274-305)
 *   moe_bind_layer   -> _unpack_tensors(_readback_device(...), metadata["tensors"])
 *                       offload_runtime/executors/_common.py:20-58, without the
 *                       device->host readback: weights stay in HBM
 *   moe_plan_create  -> GLM4MoeExecutor.__init__ / Qwen3NextExecutor.__init__
 *                       config parsing (glm4_moe.py:70-84, qwen3_next.py:105-133)
 *   moe_rt_*         -> CUDABackend (offload_runtime/backends/cuda_backend.py:35-128)
 */
#ifndef MOE_SM100_H_
#define MOE_SM100_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ----------------------------------------------------------------- status */
enum {
  MOE_OK = 0,
  MOE_ERR_INVALID = 1,        /* bad argument (ValueError in the reference)          */
  MOE_ERR_CUDA = 2,           /* CUDA runtime/driver error (RuntimeError)            */
  MOE_ERR_UNSUPPORTED = 3,    /* shape or format outside what the kernels cover      */
  MOE_ERR_MISSING_TENSOR = 4, /* a required layer tensor is absent (KeyError)        */
  MOE_ERR_WORKSPACE = 5,      /* workspace too small                                 */
  MOE_ERR_NOT_BOUND = 6,      /* forward before moe_bind_layer                       */
  MOE_ERR_DEVICE = 7,         /* a kernel reported an error (bad tile / route)       */
  MOE_ERR_TIMEOUT = 8,        /* a bounded device-side wait ran out of time          */
  MOE_ERR_RANGE = 9           /* weight value not representable in the packed format */
};

/* router scoring */
enum {
  MOE_SCORE_SOFTMAX = 0, /* softmax(logits (+ bias)), rank + weight by prob: the
                            reference rule (glm4_moe.py:181-195, qwen3_next.py:278-289) */
  MOE_SCORE_SIGMOID = 1  /* HF GLM-4.x: sigmoid(logits); select on score + bias;
                            weights are the unbiased scores                           */
};

/* on-device weight format */
enum {
  MOE_WEIGHTS_F16 = 0,     /* 16-bit expert weights (bf16 values re-encoded as f16)  */
  MOE_WEIGHTS_INT8_PC = 1  /* int8 per output row + scale (fp16 in the blob)          */
};

typedef struct MoePlan MoePlan;

/* n_experts = 0 (with top_k = 0, no bias / gate / expert range) makes a dense
 * MLP plan: the MLP of GLM-4 first_k_dense_replace layers
 * (offload_runtime/executors/glm4_moe.py:166-172, _dense_mlp_block), whose
 * mlp.{gate,up,down}_proj weights bind as a shared expert of shared_inter
 * (= intermediate_size) columns; moe_forward then returns x + MLP(rms_norm(x)).
 * moe_route and moe_ep_* refuse dense plans.
 *
 * Shape limits (moe_plan_create refuses others with MOE_ERR_UNSUPPORTED /
 * MOE_ERR_INVALID): hidden, inter and shared_inter multiples of 16 (16-byte
 * rows for TMA and the vector loads; every released GLM-4 and Qwen3 MoE model
 * qualifies, the reference's hidden-8 toy models in its integration tests do
 * not); n_experts <= 1024; 1 <= top_k <= min(32, n_experts). */
typedef struct MoeConfig {
  int32_t hidden;                /* H  (hidden_size)                                  */
  int32_t n_experts;             /* E  (n_routed_experts / num_experts)               */
  int32_t top_k;                 /* K  (num_experts_per_tok)                          */
  int32_t inter;                 /* I  (moe_intermediate_size)                        */
  int32_t shared_inter;          /* SI (shared expert intermediate; 0 = none)         */
  int32_t score_func;            /* MOE_SCORE_*                                       */
  int32_t norm_topk_prob;        /* renormalise the top-k weights                     */
  int32_t use_bias;              /* add mlp.gate.e_score_correction_bias if bound     */
  int32_t has_shared_gate;       /* Qwen3 sigmoid(h . w_gate) on the shared expert    */
  int32_t weight_format;         /* MOE_WEIGHTS_*                                     */
  float routed_scaling_factor;   /* 2.5 for GLM-4.x, 1.0 for Qwen3                    */
  float rms_norm_eps;            /* post_attention_layernorm epsilon                  */
  int32_t max_tokens;            /* largest T a forward may be called with            */
  int32_t expert_begin;          /* locally resident routed experts [begin, end);    */
  int32_t expert_end;            /*   0,0 = all (expert parallel: this rank's share)  */
  int32_t device;                /* CUDA device ordinal                               */
} MoeConfig;

/* One entry of LayerSpec.metadata["tensors"]
 * (offload_runtime/loader/huggingface.py:492-506, 560-575). */
typedef struct MoeTensorDesc {
  const char* name;   /* e.g. "mlp.experts.3.gate_proj.weight"; a "model.layers.N."
                         prefix is accepted; scales of int8 tensors are named
                         "<weight name>_scale" (fp16, one per output row)        */
  const char* dtype;  /* "float32" | "float16" | "bfloat16" | "int8"              */
  int64_t shape[2];
  int32_t ndim;
  int64_t offset;     /* byte offset inside the layer blob                        */
  int64_t nbytes;
} MoeTensorDesc;

/* ------------------------------------------------------------ plan / bind */
int moe_plan_create(const MoeConfig* cfg, MoePlan** out_plan);
int moe_plan_destroy(MoePlan* plan);

/* Pack the MoE tensors of one layer blob (already in device memory) into the
 * plan's HBM-resident layout.  The blob may be freed afterwards.  Tensors that
 * are not part of the MoE block (attention, input norm) are ignored. */
int moe_bind_layer(MoePlan* plan, const void* blob_dev, uint64_t blob_bytes,
                   const MoeTensorDesc* descs, int32_t n_descs, void* stream);

/* Bytes of device memory the plan holds for packed weights. */
uint64_t moe_plan_weight_bytes(const MoePlan* plan);

/* ---------------------------------------------------------------- compute */
/* Scratch bytes a forward / route of T tokens needs (256-byte aligned base). */
uint64_t moe_workspace_bytes(const MoePlan* plan, int32_t T);

/* out[T,H] = x + MoE(rms_norm(x)) on fp32 device buffers (x and out may not alias). */
int moe_forward(MoePlan* plan, const float* x_dev, float* out_dev, int32_t T,
                void* workspace, uint64_t workspace_bytes, void* stream);

/* moe_forward plus device time per stage, measured with CUDA events on `stream`:
 * stage_ms[0] route (RMSNorm, router, top-k, permutation + dispatch gather),
 * stage_ms[1] gate/up grouped GEMM, stage_ms[2] down grouped GEMM,
 * stage_ms[3] combine.  Synchronises `stream` before returning. */
int moe_forward_timed(MoePlan* plan, const float* x_dev, float* out_dev, int32_t T,
                      void* workspace, uint64_t workspace_bytes, float* stage_ms, void* stream);

/* Size of the library-owned scratch used by moe_forward_static_scratch. */
#define MOE_STATIC_SCRATCH_BYTES (32u * 1024u * 1024u)

/* moe_forward for callers that cannot allocate device memory (no counterpart in
 * the reference).  Some callers only own the buffers they pass in: a Go / Java /
 * C host reached through a thin FFI, a process whose memory pool has already
 * claimed the GPU, or a serving loop that must not call cudaMalloc because it
 * synchronises the device.  This entry point allocates nothing: it runs the same
 * kernels as moe_forward with a 32 MiB scratch array that lives in the library
 * (MOE_STATIC_SCRATCH_BYTES; every GPU that loads the library holds it until the
 * process exits).
 *   - The caller passes x and out as for moe_forward.
 *   - The first call on a device looks up the scratch's device address (once per
 *     device, with the plan's device current); make that first call before any
 *     stream capture.  The calling thread's current device is the same after
 *     the call as before it.
 *   - Dense-MLP plans (n_experts = 0) run here as through moe_forward.
 *   - A T whose moe_workspace_bytes(T) exceeds MOE_STATIC_SCRATCH_BYTES is
 *     rejected with MOE_ERR_WORKSPACE (for the GLM-4.7 shape, T <= 64 fits).
 *   - All calls in the process share the one scratch array and it keeps the last
 *     call's contents: calls that overlap on the GPU (different streams, or
 *     different plans on the same device at the same time) race and corrupt each
 *     other's results.  Serialise them. */
int moe_forward_static_scratch(MoePlan* plan, const float* x_dev, float* out_dev, int32_t T,
                               void* stream);

/* Router + permutation only (for parity tests and expert-parallel dispatch):
 *   topk_ids [T,K] int32, topk_w [T,K] f32, expert_offsets [E+1] int32,
 *   perm [T*K] int32 with perm[r] = t*K + slot listing rows expert-major,
 *   tokens ascending inside an expert.  Any output pointer may be NULL. */
int moe_route(MoePlan* plan, const float* x_dev, int32_t T, int32_t* topk_ids, float* topk_w,
              int32_t* expert_offsets, int32_t* perm, void* workspace,
              uint64_t workspace_bytes, void* stream);

/* ------------------------------------------------------- expert parallelism
 * New in this build (the reference runs one process on one device): the routed
 * experts are split across ranks, one process per GPU, and the caller moves
 * rows between ranks (e.g. NCCL all-to-all over NVLink).  Create each rank's
 * plan with expert_begin/expert_end = its equal, contiguous share, and bind the
 * layer blob on every rank (each packs only its own experts; router and shared
 * expert are replicated).  Per forward of T local tokens:
 *   1. moe_ep_dispatch: route the local tokens; send_rows [T*K, H] f16 holds the
 *      normalised rows grouped by destination rank (rows for rank d are
 *      send_offsets[d] .. send_offsets[d+1]), send_experts [T*K] the expert id
 *      local to the destination, send_offsets [world+1].
 *   2. caller: exchange the per-rank counts, then rows and expert ids.
 *   3. moe_ep_experts: the resident experts on the R received rows; y_out [R, H]
 *      f16 answers received row r in place.
 *   4. caller: send the y rows back (reverse exchange); they arrive in send order.
 *   5. moe_ep_shared (any time after step 1) and moe_ep_combine:
 *      out = x + sum_k w * y + shared expert.
 * Steps 1, 5 share one workspace of moe_workspace_bytes(plan, T) that must be
 * left untouched in between; step 3 uses moe_ep_workspace_bytes(plan, R). */
int moe_ep_dispatch(MoePlan* plan, const float* x_dev, int32_t T, void* send_rows,
                    int32_t* send_experts, int32_t* send_offsets, void* workspace,
                    uint64_t workspace_bytes, void* stream);
uint64_t moe_ep_workspace_bytes(const MoePlan* plan, int32_t R);
int moe_ep_experts(MoePlan* plan, const void* recv_rows, const int32_t* recv_experts, int32_t R,
                   void* y_out, void* workspace, uint64_t workspace_bytes, void* stream);
int moe_ep_shared(MoePlan* plan, int32_t T, void* workspace, uint64_t workspace_bytes,
                  void* stream);
int moe_ep_combine(MoePlan* plan, const float* x_dev, int32_t T, const void* y_back,
                   float* out_dev, void* workspace, uint64_t workspace_bytes, void* stream);

/* Fixed-capacity exchange (no host synchronisation; for small batches).  Every
 * rank sends every other rank exactly `cap` rows, so the exchange sizes are known
 * in advance and no counts cross first: one all-to-all of equal splits each way,
 * which a caller may also capture in a CUDA graph.  All ranks use the same cap,
 * at least moe_ep_capacity(plan, T) of their largest T (T * min(top_k, experts
 * per rank): no rank can then overflow a destination's share).
 *   1. moe_ep_dispatch_padded: route; send_rows [world*cap, H + 8] f16, rows
 *      [d*cap, (d+1)*cap) for rank d: H normalised values, then a 16-byte tail
 *      whose first int32 is the expert id local to d, or -1 for an unused row.
 *      Writes every row's tail (T = 0 included: all unused).  Workspace as for
 *      moe_ep_dispatch.
 *   2. caller: all-to-all of send_rows in equal splits of cap rows.
 *   3. moe_ep_experts_padded: the resident experts on the world*cap received rows
 *      (unused rows skipped); y_out [world*cap, H] f16 answers row r in place
 *      (unused rows untouched).  Workspace moe_ep_padded_workspace_bytes(plan, cap).
 *   4. caller: all-to-all of y_out back, equal splits of cap rows.
 *   5. moe_ep_shared and moe_ep_combine as above, y_back [world*cap, H]. */
int32_t moe_ep_capacity(const MoePlan* plan, int32_t T);
int moe_ep_dispatch_padded(MoePlan* plan, const float* x_dev, int32_t T, int32_t cap,
                           void* send_rows, void* workspace, uint64_t workspace_bytes,
                           void* stream);
uint64_t moe_ep_padded_workspace_bytes(const MoePlan* plan, int32_t cap);
int moe_ep_experts_padded(MoePlan* plan, const void* recv_rows, int32_t cap, void* y_out,
                          void* workspace, uint64_t workspace_bytes, void* stream);

/* Token-replicated exchange (no host synchronisation; decode batches on many
 * ranks).  Instead of sending one row per routed slot to the slot's owner, every
 * rank sends its whole batch once to every rank (an all-gather of fixed-size token
 * records), each rank applies its resident experts to the slots of all gathered
 * tokens that route to them and writes one fp32 partial sum per token, and a
 * reduce-scatter (sum) brings each rank the total for its own tokens.  Bytes moved
 * per rank do not grow with top_k or with padding to a capacity: world * cap token
 * records in, world * cap fp32 rows out.  All ranks use the same cap >= their T.
 *   1. moe_ep_token_pack: route; send_rows [cap, moe_ep_token_row_halves(plan)]
 *      f16 token records: H normalised values, then the token's top_k global
 *      expert ids (int32) and routing weights (fp32), zero-padded to 16 bytes;
 *      records T..cap-1 carry id -1 in every slot.  Workspace as moe_ep_dispatch.
 *   2. caller: all-gather of the records -> recv_rows [world*cap, ...] (rank order).
 *   3. moe_ep_experts_gathered(rows = world*cap): partial_out [rows, H] fp32, row t
 *      = sum over the slots of record t routed to this rank's experts of w * y
 *      (slot order), zero where there is none.  Workspace
 *      moe_ep_gathered_workspace_bytes(plan, rows).
 *   4. caller: reduce-scatter (sum) of partial_out -> partial [cap, H] fp32.
 *   5. moe_ep_shared (any time after step 1) and moe_ep_combine_partial:
 *      out = x + (partial + shared expert), over the first T rows of partial. */
int32_t moe_ep_token_row_halves(const MoePlan* plan);
int moe_ep_token_pack(MoePlan* plan, const float* x_dev, int32_t T, int32_t cap, void* send_rows,
                      void* workspace, uint64_t workspace_bytes, void* stream);
uint64_t moe_ep_gathered_workspace_bytes(const MoePlan* plan, int32_t rows);
int moe_ep_experts_gathered(MoePlan* plan, const void* recv_rows, int32_t rows, float* partial_out,
                            void* workspace, uint64_t workspace_bytes, void* stream);
int moe_ep_combine_partial(MoePlan* plan, const float* x_dev, int32_t T, const float* partial,
                           float* out_dev, void* workspace, uint64_t workspace_bytes, void* stream);

/* Token-replicated exchange over peer memory (no counterpart in the reference; no
 * collective library): the same records and partial sums as above, but the packing
 * and partial-sum kernels store them straight into the other GPUs' buffers over
 * NVLink and publish an epoch flag there, and a bounded wait kernel stands in for
 * each collective.  Per rank, allocated once with moe_rt_malloc (cudaMalloc'd, so
 * that moe_rt_ipc_get_handle works) and mapped on every other rank with
 * moe_rt_ipc_open_handle:
 *   recv   [world*cap, moe_ep_token_row_halves(plan)] f16, records of rank r at rows
 *          [r*cap, (r+1)*cap)
 *   part   [world, cap, H] fp32, rank r's partial sums for this rank's tokens in [r]
 *   flags  [2, world] int32, zeroed once: [0][r] records of rank r, [1][r] its
 *          partials, each the epoch of the last forward whose data is complete
 *   done   2 int32 on this rank's device, zeroed once (launch counters)
 * The peer arrays hold world device pointers, index d = rank d's buffer as mapped
 * here (d == rank: the local one).  One forward, epoch e = 1, 2, ... the same on
 * every rank, all on one stream:
 *   1. moe_ep_p2p_pack(x, T, cap, peer_recv, peer_flags, e, done + 0)
 *   2. moe_ep_p2p_wait(flags + 0, world, e)         every rank's records arrived
 *   3. moe_ep_p2p_experts(recv, cap, peer_part, peer_flags, e, done + 1)
 *   4. moe_ep_p2p_wait(flags + world, world, e)     every rank's partials arrived
 *   5. moe_ep_shared (any time after step 1) and moe_ep_p2p_combine(x, T, part):
 *      out = x + sum over source ranks (rank order) of part + shared expert.
 * Workspaces: steps 1, 5 as moe_ep_dispatch; step 3 moe_ep_gathered_workspace_bytes(
 * plan, world*cap).  A wait that runs out (a peer stopped, or is out of step)
 * returns with MOE_ERR_TIMEOUT at the next moe_status; all ranks must use the same
 * cap and epochs.  Ranks on one GPU are not supported (each wait needs the other
 * ranks' kernels running at the same time on their own GPUs). */
int moe_ep_p2p_pack(MoePlan* plan, const float* x_dev, int32_t T, int32_t cap, int32_t rank,
                    int32_t world, void* const* peer_recv, int32_t* const* peer_flags, int32_t epoch,
                    int32_t* done, void* workspace, uint64_t workspace_bytes, void* stream);
int moe_ep_p2p_wait(MoePlan* plan, const int32_t* flags, int32_t world, int32_t epoch,
                    int64_t limit_cycles, void* stream);
int moe_ep_p2p_experts(MoePlan* plan, const void* recv_rows, int32_t cap, int32_t rank,
                       int32_t world, float* const* peer_part, int32_t* const* peer_flags,
                       int32_t epoch, int32_t* done, void* workspace, uint64_t workspace_bytes,
                       void* stream);
int moe_ep_p2p_combine(MoePlan* plan, const float* x_dev, int32_t T, const float* part,
                       int32_t cap, int32_t world, float* out_dev, void* workspace,
                       uint64_t workspace_bytes, void* stream);

/* Synchronise `stream`, then read and clear the device error word of the plan.
 * Returns MOE_OK, MOE_ERR_TIMEOUT (a bounded wait ran out), MOE_ERR_RANGE (an f16
 * activation or expert output overflowed) or MOE_ERR_DEVICE. */
int moe_status(MoePlan* plan, void* stream);

/* Failure-path check (no counterpart in the reference): launch a one-thread kernel
 * that waits, with the same bounded mbarrier wait every kernel here uses, on a
 * barrier nothing arrives at, so the wait gives up after limit_cycles (<= 2e9,
 * about one second) and records a timeout in the plan's device error word; the
 * next moe_status returns MOE_ERR_TIMEOUT and the context stays usable. */
int moe_wait_probe(MoePlan* plan, int64_t limit_cycles, void* stream);

const char* moe_last_error(void);
const char* moe_version(void);

/* --------------------------------------------------- GLM-4 MoE attention
 * Replaces GLM4MoeExecutor._attention_block
 * (offload_runtime/executors/glm4_moe.py:112-162; helpers _common.py:73-155):
 *   x + o_proj(softmax(q k^T / sqrt(head_dim) + causal mask) v),
 * q, k, v = rms_norm(x, input_layernorm.weight) . W^T (+ bias), per-head RMS norm
 * of q and k times q_norm / k_norm when bound, rotate-half RoPE on the first
 * rotary_dim dims at positions 0..T-1, grouped-query heads (heads / kv_heads
 * query heads per kv head), the whole sequence at once as the reference does.
 * Weights are packed to f16 at bind (bf16-valued weights exactly; values beyond
 * +-65504 give MOE_ERR_RANGE); q / k / v / P are f16 tensor-core operands with
 * fp32 accumulation, softmax and norms in fp32.  head_dim 64 or 128; hidden a
 * multiple of 64.  Tensors are taken from the layer blob by name
 * (self_attn.{q,k,v,o}_proj.weight, self_attn.{q,k,v}_proj.bias,
 * self_attn.{q,k}_norm.weight, input_layernorm.weight; a model.layers.N.
 * prefix is accepted); biases and the q/k norms are optional. */
typedef struct MoeAttnConfig {
  int32_t hidden;       /* hidden_size                                          */
  int32_t heads;        /* num_attention_heads                                  */
  int32_t kv_heads;     /* num_key_value_heads                                  */
  int32_t head_dim;     /* 64 or 128                                            */
  int32_t rotary_dim;   /* int(head_dim * partial_rotary_factor), even           */
  float rope_theta;     /* rope_theta                                           */
  float rms_norm_eps;   /* rms_norm_eps (input norm and q/k norms)              */
  int32_t max_tokens;   /* largest sequence a forward may be called with        */
  int32_t device;       /* CUDA device ordinal                                  */
} MoeAttnConfig;

typedef struct MoeAttn MoeAttn;

int moe_attn_create(const MoeAttnConfig* cfg, MoeAttn** out);
int moe_attn_destroy(MoeAttn* attn);
/* Pack the attention tensors of a device-resident layer blob (metadata["tensors"]
 * entries, as for moe_bind_layer).  Synchronises `stream`. */
int moe_attn_bind(MoeAttn* attn, const void* blob_dev, uint64_t blob_bytes,
                  const MoeTensorDesc* descs, int32_t n_descs, void* stream);
uint64_t moe_attn_weight_bytes(const MoeAttn* attn);
uint64_t moe_attn_workspace_bytes(const MoeAttn* attn, int32_t T);
/* out[T,H] = x + attention(x); fp32, 16-byte aligned, x and out distinct. */
int moe_attn_forward(MoeAttn* attn, const float* x_dev, float* out_dev, int32_t T,
                     void* workspace, uint64_t workspace_bytes, void* stream);
/* As moe_status, for the attention kernels' device error word. */
int moe_attn_status(MoeAttn* attn, void* stream);

/* ------------------------------------------- runtime (CUDABackend, ctypes) */
int moe_rt_device_count(int32_t* count);
int moe_rt_set_device(int32_t device);
/* *can_access = 1 when `device` can map the memory of `peer`
 * (cudaDeviceCanAccessPeer); backs CUDABackend.supports_peer_to_peer. */
int moe_rt_can_access_peer(int32_t device, int32_t peer, int32_t* can_access);
int moe_rt_malloc(uint64_t nbytes, void** dev_ptr);
int moe_rt_free(void* dev_ptr);
/* CUDA IPC of a moe_rt_malloc'd buffer (64-byte handle) for the peer-memory exchange. */
int moe_rt_ipc_get_handle(const void* dev_ptr, void* handle);
int moe_rt_ipc_open_handle(const void* handle, void** dev_ptr);
int moe_rt_ipc_close_handle(void* dev_ptr);
int moe_rt_malloc_host(uint64_t nbytes, void** host_ptr);
int moe_rt_free_host(void* host_ptr);
int moe_rt_stream_create(void** stream);        /* non-blocking stream */
int moe_rt_stream_destroy(void* stream);
int moe_rt_memcpy_h2d_async(void* dst_dev, const void* src_host, uint64_t nbytes, void* stream);
int moe_rt_memcpy_d2h_async(void* dst_host, const void* src_dev, uint64_t nbytes, void* stream);
int moe_rt_memcpy_d2d_async(void* dst_dev, const void* src_dev, uint64_t nbytes, void* stream);
int moe_rt_event_record(void* stream, void** event); /* creates + records */
int moe_rt_event_destroy(void* event);
int moe_rt_stream_wait_event(void* stream, void* event);
int moe_rt_stream_synchronize(void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MOE_SM100_H_ */
