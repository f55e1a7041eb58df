// C ABI of libmoe_sm100 (declarations and reference citations: include/moe_sm100.h).
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "moe_internal.h"

namespace moe {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

static int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

static int cuda_fail(cudaError_t st, const char* what) {
  return fail(MOE_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(st));
}

#define MOE_CUDA(call)                                  \
  do {                                                  \
    cudaError_t st_ = (call);                           \
    if (st_ != cudaSuccess) return cuda_fail(st_, #call); \
  } while (0)

static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// ------------------------------------------------------------ tensor maps
static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool make_tmap_2d(CUtensorMap* map, const void* base, bool int8, uint64_t inner, uint64_t rows,
                  uint32_t box_inner, uint32_t box_rows, bool swizzle128, std::string* err) {
  auto fn = get_encode_fn();
  if (!fn) {
    *err = "cuTensorMapEncodeTiled unavailable from the driver";
    return false;
  }
  if (rows == 0) rows = 1;  // empty operand: never read, but the map must encode
  const uint64_t esize = int8 ? 1 : 2;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {inner * esize};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, int8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[160];
    snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (%d): inner=%llu rows=%llu", (int)r,
             (unsigned long long)inner, (unsigned long long)rows);
    *err = buf;
    return false;
  }
  return true;
}

// ------------------------------------------------------------ workspace
static int pick_bn(int T) {
  if (T <= 16) return 16;
  if (T <= 32) return 32;
  if (T <= 64) return 64;
  if (T <= 128) return 128;
  return 256;
}

// Workspace for `rows` (tokens or received rows) x `k` routed slots over
// `groups` expert groups; `shared_rows` rows for the shared expert; the router
// buffers only when `router`.
static WsLayout ws_layout_general(const Plan& p, int rows, int k, int groups, int shared_rows,
                                  int bn, bool router, bool ybuf = false) {
  WsLayout L{};
  const int T = rows;
  const size_t R = static_cast<size_t>(T) * k;
  const int E = groups;
  const int TS = shared_rows;
  L.bn = bn;
  L.nchunks = (T + kPermChunk - 1) / kPermChunk;
  const int mt1 = (2 * p.I + kBM - 1) / kBM;
  const int mt2 = (p.H + kBM - 1) / kBM;
  const int mt1s = (p.SI > 0 && TS > 0) ? (2 * p.SI + kBM - 1) / kBM : 0;
  const int ntr = static_cast<int>((R + L.bn - 1) / L.bn) + static_cast<int>(R < (size_t)E ? R : E);
  const int nts = (p.SI > 0 && TS > 0) ? (TS + L.bn - 1) / L.bn : 0;
  L.max_tiles1 = ntr * mt1 + nts * mt1s;
  L.max_tiles2 = ntr * mt2 + nts * mt2;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    size_t at = o;
    o = align256(o + bytes);
    return at;
  };
  L.h16 = take(static_cast<size_t>(router ? T : TS) * p.H * 2);
  L.xg = take(R * p.H * 2);
  L.act = take(R * p.I * 2);
  L.act_s = take(static_cast<size_t>(TS) * p.SI * 2);
  L.y = take((router || ybuf) ? R * p.H * 2 : 0);  // routed expert outputs, f16, dispatch order
  L.y_s = take(p.SI > 0 ? static_cast<size_t>(TS) * p.H * 4 : 0);
  if (router) {
    const RouterGeom g = router_geometry(p, T);
    // prefill batches may route on the tensor cores: one logit plane per K split
    const size_t planes = route_uses_tail(p, T) ? 1 : kRouterMaxSplit;
    L.logits = take(planes * T * p.router_rows * 4);
    L.part = take(g.splits > 1 ? static_cast<size_t>(g.splits) * T * p.router_rows * 4 : 0);
    L.ss_part = take(static_cast<size_t>(g.rx) * g.splits * T * 4);
    L.rms = take(static_cast<size_t>(T) * 4);
    L.counters = take(static_cast<size_t>(g.rx) * g.tz * 4);
    L.ids = take(R * 4);
    L.wts = take(R * 4);
    L.sgate = take(static_cast<size_t>(T) * 4);
    const bool prefill = !route_uses_tail(p, T);
    L.cand = take(prefill ? static_cast<size_t>(T) * kCandMax * 4 : 0);
    L.ncand = take(prefill ? static_cast<size_t>(T) * 4 : 0);
    L.exact = take(prefill ? static_cast<size_t>(T) * (kCandMax + 1) * 4 : 0);
  } else if (p.E == 0) {
    L.rms = take(static_cast<size_t>(T) * 4);  // dense MLP: per-token rms of the prologue
  }
  L.bm = take(static_cast<size_t>(L.nchunks) * E * 32 * 4);
  L.hist = take(static_cast<size_t>(L.nchunks) * E * 4);
  L.base = take(static_cast<size_t>(L.nchunks) * E * 4);
  L.offsets = take(static_cast<size_t>(E + 1) * 4);
  L.perm = take(R * 4);
  L.slot_row = take(R * 4);
  // split-K is used only for 16-token tiles when a list has fewer than four
  // waves of tiles, so its scratch is bounded by 4 * SMs tiles of kMaxKSplit partials
  L.max_split_tiles = (L.bn == kSplitTileRows) ? 4 * p.num_sms : 0;
  L.tile_pre = take(static_cast<size_t>(2) * (E + 1) * 4);
  L.tile_info = take(32);
  L.kpart = take(static_cast<size_t>(L.max_split_tiles) * kMaxKSplit * kBM * kSplitTileRows * 4);
  L.kcount1 = take(static_cast<size_t>(L.max_split_tiles) * 4);
  L.kcount2 = take(static_cast<size_t>(L.max_split_tiles) * 4);
  L.total = o;
  return L;
}

// 16-bit prefill batches whose experts average at most ~176 tokens take 192-token
// tiles instead of 256: such a GEMM is bound by streaming the expert weights, and
// the narrower token tile leaves room for a fifth stage of weights in flight while
// most experts still fit in one tile (each extra tile re-reads the weights).
#ifndef MOE_PREFILL_BN_NARROW
#define MOE_PREFILL_BN_NARROW 1
#endif
static int prefill_bn(const Plan& p, int T) {
  const int bn = pick_bn(T);
  if (MOE_PREFILL_BN_NARROW && bn == 256 && !p.int8 && p.E > 0 &&
      static_cast<int64_t>(T) * p.K <= 176LL * p.E)
    return 192;
  return bn;
}

WsLayout ws_layout(const Plan& p, int T) {
  if (p.E == 0)  // dense MLP: normalised rows and the shared-expert GEMMs only
    return ws_layout_general(p, T, 0, 0, T, pick_bn(T), false);
  // INT8 decode batches keep token tiles of at most 64 columns, so that their
  // GEMMs take the TMEM-A path (gemm_ts): an expert sees ~T*K/E tokens, far fewer
  // than T, and the wider tiles' shared-memory A path ran ~25 % slower at T = 128.
  const int bn = (p.int8 && route_uses_tail(p, T)) ? std::min(pick_bn(T), 64) : prefill_bn(p, T);
  return ws_layout_general(p, T, p.K, p.E, p.SI > 0 ? T : 0, bn, true);
}

// Expert side of the expert-parallel path: R received rows grouped by the
// n_local resident experts, no router, no shared expert.  The token tile width
// follows the rows expected to be valid (`expect`: all R for the exact
// exchange, one rank's capacity for the fixed-capacity one), the buffers the
// worst case of R.
WsLayout ws_layout_ep_experts(const Plan& p, int R, int expect) {
  const int per_expert = (2 * expect + p.n_local - 1) / (p.n_local > 0 ? p.n_local : 1);
  return ws_layout_general(p, R, 1, p.n_local, 0, pick_bn(per_expert > 0 ? per_expert : 1), false);
}

// Expert side of the token-replicated exchange: the K slots of `rows` gathered
// token records, of which those routed to the resident experts are grouped, with
// the f16 expert outputs in grouped order (L.y).  On average a rank keeps 1/world
// of the slots; the tile width follows that, the buffers the worst case.
WsLayout ws_layout_ep_gathered(const Plan& p, int rows) {
  const int64_t kept = static_cast<int64_t>(rows) * p.K * p.n_local / std::max(p.E, 1);
  const int64_t per_expert = (2 * kept + p.n_local - 1) / std::max(p.n_local, 1);
  return ws_layout_general(p, rows, p.K, p.n_local, 0,
                           pick_bn(static_cast<int>(std::max<int64_t>(per_expert, 1))), false, true);
}

// ------------------------------------------------------------ name parsing
enum Kind { K_NONE, K_NORM, K_ROUTER, K_BIAS, K_SHARED_GATE, K_EXPERT, K_SHARED, K_DENSE };
enum Proj { P_GATE = 0, P_UP = 1, P_DOWN = 2 };

struct Parsed {
  Kind kind = K_NONE;
  int expert = -1;
  int proj = -1;
  bool scale = false;
};

static bool starts_with(const std::string& s, const char* pre) {
  return s.compare(0, strlen(pre), pre) == 0;
}

static bool parse_proj(const std::string& rest, Parsed* out) {
  static const char* names[3] = {"gate_proj.weight", "up_proj.weight", "down_proj.weight"};
  for (int i = 0; i < 3; ++i) {
    const std::string n = names[i];
    if (rest == n) {
      out->proj = i;
      return true;
    }
    if (rest == n + "_scale") {
      out->proj = i;
      out->scale = true;
      return true;
    }
  }
  return false;
}

static Parsed parse_name(const char* cname) {
  Parsed p;
  std::string n(cname ? cname : "");
  const size_t pos_norm = n.find("post_attention_layernorm.weight");
  if (pos_norm != std::string::npos && pos_norm + strlen("post_attention_layernorm.weight") == n.size()) {
    p.kind = K_NORM;
    return p;
  }
  const size_t pos = n.find("mlp.");
  if (pos == std::string::npos) return p;
  std::string s = n.substr(pos);
  if (s == "mlp.gate.weight") p.kind = K_ROUTER;
  else if (s == "mlp.gate.e_score_correction_bias") p.kind = K_BIAS;
  else if (s == "mlp.shared_expert_gate.weight") p.kind = K_SHARED_GATE;
  else if (parse_proj(s.substr(4), &p)) p.kind = K_DENSE;  // mlp.{gate,up,down}_proj (dense layers)
  else if (starts_with(s, "mlp.shared_experts.") || starts_with(s, "mlp.shared_expert.")) {
    const std::string rest = s.substr(s.find('.', 4) + 1);
    if (parse_proj(rest, &p)) p.kind = K_SHARED;
  } else if (starts_with(s, "mlp.experts.")) {
    const std::string r = s.substr(strlen("mlp.experts."));
    const size_t dot = r.find('.');
    if (dot != std::string::npos && dot > 0) {
      int e = 0;
      bool ok = true;
      for (size_t i = 0; i < dot; ++i) {
        if (r[i] < '0' || r[i] > '9') ok = false;
        else e = e * 10 + (r[i] - '0');
      }
      if (ok && parse_proj(r.substr(dot + 1), &p)) {
        p.kind = K_EXPERT;
        p.expert = e;
      }
    }
  }
  return p;
}

static int parse_dtype(const char* d) {
  std::string s(d ? d : "");
  if (s == "float32" || s == "<f4" || s == "f4") return SRC_F32;
  if (s == "float16" || s == "<f2" || s == "f2") return SRC_F16;
  if (s == "bfloat16" || s == "bf16") return SRC_BF16;
  if (s == "int8" || s == "|i1" || s == "i1") return SRC_I8;
  return -1;
}

static size_t dtype_size(int d) { return d == SRC_F32 ? 4 : (d == SRC_I8 ? 1 : 2); }

// One thread waits, with the bounded wait every kernel here uses, on an mbarrier
// that nothing ever arrives at.  The wait gives up after `limit` cycles and the
// kernel records a timeout in the plan's error word and returns: the failure
// path of a stuck pipeline, without a fault and without a stuck GPU.
__global__ void wait_probe_kernel(int* err, long long limit) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !mbar_wait_bounded(&bar, 0, &abort_flag, limit))
    record_error(err, DEV_TIMEOUT_FULL);
}

}  // namespace moe

// ====================================================================== C ABI
using namespace moe;

extern "C" {

const char* moe_last_error(void) { return g_last_error.c_str(); }
const char* moe_version(void) { return "moe_sm100 0.1 (sm_100a, tcgen05)"; }

int moe_plan_create(const MoeConfig* cfg, MoePlan** out_plan) {
  if (!cfg || !out_plan) return fail(MOE_ERR_INVALID, "null argument");
  const MoeConfig& c = *cfg;
  if (c.hidden <= 0 || c.hidden % 16 != 0)
    return fail(MOE_ERR_UNSUPPORTED, "hidden must be a positive multiple of 16");
  // n_experts == 0: the dense MLP of a first_k_dense_replace layer
  // (glm4_moe.py:166-172), computed as a shared expert of shared_inter columns
  const bool dense = c.n_experts == 0;
  if (dense) {
    if (c.top_k != 0 || c.use_bias || c.has_shared_gate || c.expert_begin || c.expert_end)
      return fail(MOE_ERR_INVALID,
                  "a dense MLP plan (n_experts = 0) takes top_k = 0, no bias, gate or expert range");
    if (c.shared_inter <= 0)
      return fail(MOE_ERR_INVALID, "a dense MLP plan needs shared_inter = intermediate_size");
  }
  if (c.inter < 0 || c.inter % 16 != 0 || (!dense && c.inter == 0))
    return fail(MOE_ERR_UNSUPPORTED, "moe_intermediate_size must be a positive multiple of 16");
  if (c.shared_inter < 0 || c.shared_inter % 16 != 0)
    return fail(MOE_ERR_UNSUPPORTED, "shared intermediate size must be a multiple of 16");
  if (c.n_experts < 0 || c.n_experts > 1024)
    return fail(MOE_ERR_UNSUPPORTED, "n_experts must be in [0, 1024]");
  if (!dense && (c.top_k <= 0 || c.top_k > kMaxTopK || c.top_k > c.n_experts))
    return fail(MOE_ERR_INVALID, "top_k must be in [1, min(32, n_experts)]");
  if (c.score_func != MOE_SCORE_SOFTMAX && c.score_func != MOE_SCORE_SIGMOID)
    return fail(MOE_ERR_INVALID, "unknown score_func");
  if (c.weight_format != MOE_WEIGHTS_F16 && c.weight_format != MOE_WEIGHTS_INT8_PC)
    return fail(MOE_ERR_INVALID, "unknown weight_format");
  if (c.max_tokens <= 0) return fail(MOE_ERR_INVALID, "max_tokens must be positive");
  if (c.has_shared_gate && c.shared_inter == 0)
    return fail(MOE_ERR_INVALID, "shared gate requires a shared expert");
  int eb = c.expert_begin, ee = c.expert_end;
  if (eb == 0 && ee == 0) ee = c.n_experts;
  if (!dense && (eb < 0 || ee > c.n_experts || eb >= ee)) return fail(MOE_ERR_INVALID, "bad expert range");
  if (!dense && (c.n_experts % (ee - eb) != 0 || eb % (ee - eb) != 0))
    return fail(MOE_ERR_INVALID,
                "expert share must be one of n_experts / share equal contiguous ranges");

  MOE_CUDA(cudaSetDevice(c.device));
  MoePlan* plan = new MoePlan();
  Plan& p = plan->p;
  p.cfg = c;
  p.device = c.device;
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, c.device);
  p.num_sms = sms > 0 ? sms : 148;
  p.E = c.n_experts;
  p.K = c.top_k;
  p.H = c.hidden;
  p.I = c.inter > 0 ? c.inter : c.shared_inter;  // a dense plan has no routed I
  p.SI = c.shared_inter;
  p.e_begin = eb;
  p.e_end = ee;
  p.n_local = ee - eb;
  p.router_rows = p.E + (c.has_shared_gate ? 1 : 0);
  p.int8 = c.weight_format == MOE_WEIGHTS_INT8_PC;
  cudaError_t st = cudaMalloc(&p.d_err, sizeof(int));
  if (st == cudaSuccess) st = cudaMemset(p.d_err, 0, sizeof(int));
  if (st != cudaSuccess) {
    delete plan;
    return cuda_fail(st, "cudaMalloc(error word)");
  }
  *out_plan = plan;
  return MOE_OK;
}

int moe_plan_destroy(MoePlan* plan) {
  if (!plan) return MOE_OK;
  cudaSetDevice(plan->p.device);
  if (plan->p.weights_alloc) cudaFree(plan->p.weights_alloc);
  if (plan->p.d_err) cudaFree(plan->p.d_err);
  delete plan;
  return MOE_OK;
}

uint64_t moe_plan_weight_bytes(const MoePlan* plan) { return plan ? plan->p.weights_bytes : 0; }

int moe_bind_layer(MoePlan* plan, const void* blob_dev, uint64_t blob_bytes,
                   const MoeTensorDesc* descs, int32_t n_descs, void* stream) {
  if (!plan || !blob_dev || !descs || n_descs <= 0) return fail(MOE_ERR_INVALID, "null argument");
  Plan& p = plan->p;
  MOE_CUDA(cudaSetDevice(p.device));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int E = p.E, H = p.H, I = p.I, SI = p.SI, NL = p.n_local;

  struct Src {
    const char* ptr = nullptr;
    int dtype = -1;
  };
  Src norm, router, bias, sgate;
  std::vector<Src> ex(static_cast<size_t>(NL) * 3), exs(static_cast<size_t>(NL) * 3);
  Src sh[3], shs[3];
  const char* base = static_cast<const char*>(blob_dev);

  for (int i = 0; i < n_descs; ++i) {
    const MoeTensorDesc& d = descs[i];
    const Parsed pn = parse_name(d.name);
    if (pn.kind == K_NONE) continue;
    const int dt = parse_dtype(d.dtype);
    if (dt < 0) return fail(MOE_ERR_UNSUPPORTED, std::string("unsupported dtype for ") + d.name);
    if (d.offset < 0 || d.nbytes < 0 || static_cast<uint64_t>(d.offset + d.nbytes) > blob_bytes)
      return fail(MOE_ERR_INVALID, std::string("tensor outside the blob: ") + d.name);
    int64_t numel = 1;
    for (int k = 0; k < d.ndim && k < 2; ++k) numel *= d.shape[k];
    if (d.ndim < 1 || d.ndim > 2 || numel * static_cast<int64_t>(dtype_size(dt)) != d.nbytes)
      return fail(MOE_ERR_INVALID, std::string("shape / nbytes mismatch for ") + d.name);
    const int64_t r0 = d.shape[0], c0 = d.ndim == 2 ? d.shape[1] : 1;
    auto need = [&](int64_t rows, int64_t cols) {
      return (d.ndim == 2 && r0 == rows && c0 == cols) || (d.ndim == 1 && cols == 1 && r0 == rows);
    };
    Src src{base + d.offset, dt};
    switch (pn.kind) {
      case K_NORM:
        if (!need(H, 1)) return fail(MOE_ERR_INVALID, "post_attention_layernorm.weight shape");
        norm = src;
        break;
      case K_ROUTER:
        if (!need(E, H)) return fail(MOE_ERR_INVALID, "mlp.gate.weight must be [n_experts, hidden]");
        router = src;
        break;
      case K_BIAS:
        if (!need(E, 1)) return fail(MOE_ERR_INVALID, "e_score_correction_bias must be [n_experts]");
        bias = src;
        break;
      case K_SHARED_GATE:
        if (!(d.ndim == 2 && r0 == 1 && c0 == H) && !(d.ndim == 1 && r0 == H))
          return fail(MOE_ERR_INVALID, "mlp.shared_expert_gate.weight must be [1, hidden]");
        sgate = src;
        break;
      case K_EXPERT: {
        if (pn.expert < 0 || pn.expert >= E)
          return fail(MOE_ERR_INVALID, std::string("expert id out of range: ") + d.name);
        const int le = pn.expert - p.e_begin;
        if (le < 0 || le >= NL) break;  // not resident on this plan
        const int64_t rows = pn.proj == P_DOWN ? H : I, cols = pn.proj == P_DOWN ? I : H;
        if (pn.scale) {
          if (dt != SRC_F16 || !need(rows, 1))
            return fail(MOE_ERR_INVALID, std::string("scale must be float16 [rows]: ") + d.name);
          exs[static_cast<size_t>(le) * 3 + pn.proj] = src;
        } else {
          if (!need(rows, cols)) return fail(MOE_ERR_INVALID, std::string("expert weight shape: ") + d.name);
          ex[static_cast<size_t>(le) * 3 + pn.proj] = src;
        }
        break;
      }
      case K_DENSE:
      case K_SHARED: {
        // a dense MLP plan packs mlp.*_proj into the shared-expert slots; a MoE
        // plan packs the shared expert and ignores dense-layer names
        if ((pn.kind == K_DENSE) != (E == 0)) break;
        const int64_t rows = pn.proj == P_DOWN ? H : SI, cols = pn.proj == P_DOWN ? SI : H;
        if (SI == 0) break;
        if (pn.scale) {
          if (dt != SRC_F16 || !need(rows, 1))
            return fail(MOE_ERR_INVALID, std::string("scale must be float16 [rows]: ") + d.name);
          shs[pn.proj] = src;
        } else {
          if (!need(rows, cols)) return fail(MOE_ERR_INVALID, std::string("shared expert shape: ") + d.name);
          sh[pn.proj] = src;
        }
        break;
      }
      default: break;
    }
  }
  if (!norm.ptr) return fail(MOE_ERR_MISSING_TENSOR, "post_attention_layernorm.weight");
  if (E > 0 && !router.ptr) return fail(MOE_ERR_MISSING_TENSOR, "mlp.gate.weight");
  if (p.cfg.has_shared_gate && !sgate.ptr) return fail(MOE_ERR_MISSING_TENSOR, "mlp.shared_expert_gate.weight");
  static const char* pname[3] = {"gate_proj", "up_proj", "down_proj"};
  for (int le = 0; le < NL; ++le)
    for (int j = 0; j < 3; ++j) {
      const Src& w = ex[static_cast<size_t>(le) * 3 + j];
      if (!w.ptr) return fail(MOE_ERR_MISSING_TENSOR, "mlp.experts." + std::to_string(le + p.e_begin) + "." + pname[j] + ".weight");
      if (w.dtype == SRC_I8 && !exs[static_cast<size_t>(le) * 3 + j].ptr)
        return fail(MOE_ERR_MISSING_TENSOR, "mlp.experts." + std::to_string(le + p.e_begin) + "." + pname[j] + ".weight_scale");
      if (w.dtype == SRC_I8 && !p.int8)
        return fail(MOE_ERR_UNSUPPORTED, "int8 expert weights need weight_format = MOE_WEIGHTS_INT8_PC");
    }
  for (int j = 0; j < 3 && SI > 0; ++j) {
    if (!sh[j].ptr)
      return fail(MOE_ERR_MISSING_TENSOR, E == 0 ? std::string("mlp.") + pname[j] + ".weight"
                                                 : std::string("shared expert ") + pname[j]);
    if (sh[j].dtype == SRC_I8 && !shs[j].ptr) return fail(MOE_ERR_MISSING_TENSOR, std::string("shared expert scale ") + pname[j]);
    if (sh[j].dtype == SRC_I8 && !p.int8)
      return fail(MOE_ERR_UNSUPPORTED, "int8 shared weights need weight_format = MOE_WEIGHTS_INT8_PC");
  }

  // ---- allocate the resident layout (once per plan; reused by later binds)
  size_t o = 0;
  auto take = [&](size_t b) { size_t at = o; o = align256(o + b); return at; };
  // one expert matrix: f16 row-major, or int8 tile-major with its padding
  auto mat_bytes = [&](int m, int k) {
    return p.int8 ? i8_pad_rows(m) * i8_pad_cols(k) : static_cast<size_t>(m) * k * 2;
  };
  const size_t b13 = mat_bytes(2 * I, H), b2 = mat_bytes(H, I);
  const size_t o_w13 = take(static_cast<size_t>(NL) * b13);
  const size_t o_w2 = take(static_cast<size_t>(NL) * b2);
  const size_t o_ws13 = take(mat_bytes(2 * SI, H));
  const size_t o_ws2 = take(mat_bytes(H, SI));
  const size_t o_s13 = take(p.int8 ? static_cast<size_t>(NL) * 2 * I * 4 : 0);
  const size_t o_s2 = take(p.int8 ? static_cast<size_t>(NL) * H * 4 : 0);
  const size_t o_ss13 = take(p.int8 ? static_cast<size_t>(2) * SI * 4 : 0);
  const size_t o_ss2 = take(p.int8 && SI > 0 ? static_cast<size_t>(H) * 4 : 0);
  const size_t o_norm = take(static_cast<size_t>(H) * 4);
  const size_t o_router = take(static_cast<size_t>(p.router_rows) * H * 4);
  const size_t o_bias = take(static_cast<size_t>(E) * 4);
  const size_t o_rw16 = take(static_cast<size_t>(p.router_rows) * H * 2);
  const size_t o_flag = take(16);
  if (!p.weights_alloc) {
    MOE_CUDA(cudaMalloc(&p.weights_alloc, o));
    p.weights_bytes = o;
  }
  char* wb = static_cast<char*>(p.weights_alloc);
  p.w.w13 = wb + o_w13;
  p.w.w2 = wb + o_w2;
  p.w.ws13 = SI > 0 ? wb + o_ws13 : nullptr;
  p.w.ws2 = SI > 0 ? wb + o_ws2 : nullptr;
  p.w.s13 = p.int8 ? reinterpret_cast<float*>(wb + o_s13) : nullptr;
  p.w.s2 = p.int8 ? reinterpret_cast<float*>(wb + o_s2) : nullptr;
  p.w.ss13 = p.int8 && SI > 0 ? reinterpret_cast<float*>(wb + o_ss13) : nullptr;
  p.w.ss2 = p.int8 && SI > 0 ? reinterpret_cast<float*>(wb + o_ss2) : nullptr;
  p.w.norm_w = reinterpret_cast<float*>(wb + o_norm);
  p.w.router_w = reinterpret_cast<float*>(wb + o_router);
  p.w.bias = (bias.ptr && p.cfg.use_bias) ? reinterpret_cast<float*>(wb + o_bias) : nullptr;
  p.w.rw16 = reinterpret_cast<__half*>(wb + o_rw16);
  int* range_err = reinterpret_cast<int*>(wb + o_flag);
  int* rw16_err = range_err + 1;
  MOE_CUDA(cudaMemsetAsync(range_err, 0, 2 * sizeof(int), s));
  // int8 tiles are padded: zero the expert matrices before the packers fill them
  if (p.int8) MOE_CUDA(cudaMemsetAsync(wb + o_w13, 0, o_s13 - o_w13, s));

  // ---- pack
  MOE_CUDA(launch_to_f32(norm.ptr, norm.dtype, p.w.norm_w, H, s));
  if (E > 0) MOE_CUDA(launch_to_f32(router.ptr, router.dtype, p.w.router_w, static_cast<int64_t>(E) * H, s));
  if (sgate.ptr)
    MOE_CUDA(launch_to_f32(sgate.ptr, sgate.dtype, p.w.router_w + static_cast<size_t>(E) * H, H, s));
  if (p.w.bias) MOE_CUDA(launch_to_f32(bias.ptr, bias.dtype, p.w.bias, E, s));
  if (p.router_rows > 0)
    MOE_CUDA(launch_scale_router_weights(p.w.router_w, p.w.rw16, p.router_rows, H, rw16_err, s));
  for (int le = 0; le < NL; ++le) {
    const Src& g = ex[le * 3 + P_GATE];
    const Src& u = ex[le * 3 + P_UP];
    const Src& dn = ex[le * 3 + P_DOWN];
    char* d13 = static_cast<char*>(p.w.w13) + static_cast<size_t>(le) * b13;
    char* d2 = static_cast<char*>(p.w.w2) + static_cast<size_t>(le) * b2;
    float* s13 = p.int8 ? p.w.s13 + static_cast<size_t>(le) * 2 * I : nullptr;
    float* s2 = p.int8 ? p.w.s2 + static_cast<size_t>(le) * H : nullptr;
    if (g.dtype == SRC_I8 || u.dtype == SRC_I8) {
      if (g.dtype != SRC_I8 || u.dtype != SRC_I8) return fail(MOE_ERR_UNSUPPORTED, "gate/up must share a dtype");
      MOE_CUDA(launch_copy_i8_w13(reinterpret_cast<const int8_t*>(g.ptr), reinterpret_cast<const int8_t*>(u.ptr),
                                  reinterpret_cast<const __half*>(exs[le * 3 + P_GATE].ptr),
                                  reinterpret_cast<const __half*>(exs[le * 3 + P_UP].ptr),
                                  reinterpret_cast<int8_t*>(d13), s13, I, H, s));
    } else {
      if (g.dtype != u.dtype) return fail(MOE_ERR_UNSUPPORTED, "gate/up must share a dtype");
      MOE_CUDA(launch_pack_w13(g.ptr, u.ptr, g.dtype, d13, p.int8, s13, I, H, range_err, s));
    }
    if (dn.dtype == SRC_I8)
      MOE_CUDA(launch_copy_i8_rows(reinterpret_cast<const int8_t*>(dn.ptr),
                                   reinterpret_cast<const __half*>(exs[le * 3 + P_DOWN].ptr),
                                   reinterpret_cast<int8_t*>(d2), s2, H, I, s));
    else
      MOE_CUDA(launch_pack_rows(dn.ptr, dn.dtype, d2, p.int8, s2, H, I, range_err, s));
  }
  if (SI > 0) {
    if (sh[P_GATE].dtype == SRC_I8) {
      MOE_CUDA(launch_copy_i8_w13(reinterpret_cast<const int8_t*>(sh[P_GATE].ptr),
                                  reinterpret_cast<const int8_t*>(sh[P_UP].ptr),
                                  reinterpret_cast<const __half*>(shs[P_GATE].ptr),
                                  reinterpret_cast<const __half*>(shs[P_UP].ptr),
                                  reinterpret_cast<int8_t*>(p.w.ws13), p.w.ss13, SI, H, s));
    } else {
      MOE_CUDA(launch_pack_w13(sh[P_GATE].ptr, sh[P_UP].ptr, sh[P_GATE].dtype, p.w.ws13, p.int8,
                               p.w.ss13, SI, H, range_err, s));
    }
    if (sh[P_DOWN].dtype == SRC_I8)
      MOE_CUDA(launch_copy_i8_rows(reinterpret_cast<const int8_t*>(sh[P_DOWN].ptr),
                                   reinterpret_cast<const __half*>(shs[P_DOWN].ptr),
                                   reinterpret_cast<int8_t*>(p.w.ws2), p.w.ss2, H, SI, s));
    else
      MOE_CUDA(launch_pack_rows(sh[P_DOWN].ptr, sh[P_DOWN].dtype, p.w.ws2, p.int8, p.w.ss2, H, SI,
                                range_err, s));
  }
  int h_range[2] = {0, 0};
  MOE_CUDA(cudaMemcpyAsync(h_range, range_err, 2 * sizeof(int), cudaMemcpyDeviceToHost, s));
  MOE_CUDA(cudaStreamSynchronize(s));
  if (h_range[0]) return fail(MOE_ERR_RANGE, "an expert weight does not fit the packed format (|w| > 65504 for f16)");
  // Prefill batches pick candidate experts on the tensor cores and recompute
  // the chosen logits in fp32.  Two cases keep the fp32 CUDA-core router of
  // decode batches instead: router weights beyond |w| ~ 64 (no scaled f16
  // copy), and softmax weights without renormalisation, whose denominator
  // would carry the f16 error of every non-selected logit.
  p.router_tc = h_range[1] == 0 &&
                !(p.cfg.score_func == MOE_SCORE_SOFTMAX && !p.cfg.norm_topk_prob);

  // ---- tensor maps over the resident f16 weights (int8 tiles are fetched as
  // contiguous blocks straight from their tile-major layout)
  std::string err;
  if (!p.int8) {
    if (!make_tmap_2d(&p.tm_w13, p.w.w13, false, H, static_cast<uint64_t>(NL) * 2 * I, kBK, kBM, true, &err) ||
        !make_tmap_2d(&p.tm_w2, p.w.w2, false, I, static_cast<uint64_t>(NL) * H, kBK, kBM, true, &err))
      return fail(MOE_ERR_CUDA, err);
    if (SI > 0 &&
        (!make_tmap_2d(&p.tm_ws13, p.w.ws13, false, H, 2 * SI, kBK, kBM, true, &err) ||
         !make_tmap_2d(&p.tm_ws2, p.w.ws2, false, SI, H, kBK, kBM, true, &err)))
      return fail(MOE_ERR_CUDA, err);
  }
  if (!make_tmap_2d(&p.tm_rw16, p.w.rw16, false, static_cast<uint64_t>(H), p.router_rows,
                    kBK, kBM, true, &err))
    return fail(MOE_ERR_CUDA, err);
  p.bound = true;
  return MOE_OK;
}

uint64_t moe_workspace_bytes(const MoePlan* plan, int32_t T) {
  if (!plan || T <= 0) return 0;
  return ws_layout(plan->p, T).total;
}

static int check_call(const MoePlan* plan, int32_t T, const void* ws, uint64_t ws_bytes) {
  if (!plan) return fail(MOE_ERR_INVALID, "null plan");
  if (!plan->p.bound) return fail(MOE_ERR_NOT_BOUND, "moe_bind_layer has not been called");
  if (plan->p.n_local != plan->p.E)
    return fail(MOE_ERR_UNSUPPORTED,
                "this plan holds a share of the experts: use the moe_ep_* entry points");
  if (T < 0 || T > plan->p.cfg.max_tokens)
    return fail(MOE_ERR_INVALID, "T outside [0, max_tokens]");
  if (T == 0) return MOE_OK;
  if (!ws || (reinterpret_cast<uintptr_t>(ws) & 255))
    return fail(MOE_ERR_WORKSPACE, "workspace must be a 256-byte aligned device pointer");
  if (ws_bytes < ws_layout(plan->p, T).total) return fail(MOE_ERR_WORKSPACE, "workspace too small");
  return MOE_OK;
}

static int route_impl(Plan& p, const WsLayout& L, char* ws, const float* x, int T,
                      bool dispatch, cudaStream_t s) {
  if (p.E == 0) {  // dense MLP: normalised f16 rows, then the shared-expert tile map
    MOE_CUDA(launch_row_prep(p, L, ws, x, T, s));
    MOE_CUDA(launch_shared_tiles(p, L, ws, T, s));
    return MOE_OK;
  }
  MOE_CUDA(launch_route(p, L, ws, x, T, dispatch, s));
  return MOE_OK;
}

int moe_forward(MoePlan* plan, const float* x_dev, float* out_dev, int32_t T, void* workspace,
                uint64_t workspace_bytes, void* stream) {
  int rc = check_call(plan, T, workspace, workspace_bytes);
  if (rc != MOE_OK || T == 0) return rc;
  if (!x_dev || !out_dev) return fail(MOE_ERR_INVALID, "null x / out");
  if (x_dev == out_dev) return fail(MOE_ERR_INVALID, "x and out may not alias");
  if (misaligned16(x_dev) || misaligned16(out_dev))
    return fail(MOE_ERR_INVALID, "x and out must be 16-byte aligned");
  Plan& p = plan->p;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const WsLayout L = ws_layout(p, T);
  char* ws = static_cast<char*>(workspace);
  rc = route_impl(p, L, ws, x_dev, T, true, s);
  if (rc != MOE_OK) return rc;
  MOE_CUDA(launch_gemm(p, L, ws, false, T, s));
  MOE_CUDA(launch_gemm(p, L, ws, true,
                       GemmIO{T * p.K, T, reinterpret_cast<__half*>(ws + L.y), nullptr, p.n_local}, s));
  MOE_CUDA(launch_combine_half(p, x_dev, reinterpret_cast<const __half*>(ws + L.y),
                          reinterpret_cast<float*>(ws + L.y_s),
                          reinterpret_cast<int32_t*>(ws + L.slot_row),
                          reinterpret_cast<float*>(ws + L.wts),
                          reinterpret_cast<float*>(ws + L.sgate), out_dev, T, s));
  return MOE_OK;
}

int moe_forward_timed(MoePlan* plan, const float* x_dev, float* out_dev, int32_t T,
                      void* workspace, uint64_t workspace_bytes, float* stage_ms, void* stream) {
  int rc = check_call(plan, T, workspace, workspace_bytes);
  if (rc != MOE_OK) return rc;
  if (!x_dev || !out_dev || !stage_ms) return fail(MOE_ERR_INVALID, "null x / out / stage_ms");
  if (x_dev == out_dev) return fail(MOE_ERR_INVALID, "x and out may not alias");
  if (misaligned16(x_dev) || misaligned16(out_dev))
    return fail(MOE_ERR_INVALID, "x and out must be 16-byte aligned");
  for (int i = 0; i < 4; ++i) stage_ms[i] = 0.f;
  if (T == 0) return MOE_OK;
  Plan& p = plan->p;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const WsLayout L = ws_layout(p, T);
  char* ws = static_cast<char*>(workspace);
  cudaEvent_t ev[5];
  for (int i = 0; i < 5; ++i) MOE_CUDA(cudaEventCreate(&ev[i]));
  struct Guard {
    cudaEvent_t* e;
    ~Guard() {
      for (int i = 0; i < 5; ++i) cudaEventDestroy(e[i]);
    }
  } guard{ev};
  MOE_CUDA(cudaEventRecord(ev[0], s));
  rc = route_impl(p, L, ws, x_dev, T, true, s);
  if (rc != MOE_OK) return rc;
  MOE_CUDA(cudaEventRecord(ev[1], s));
  MOE_CUDA(launch_gemm(p, L, ws, false, T, s));
  MOE_CUDA(cudaEventRecord(ev[2], s));
  MOE_CUDA(launch_gemm(p, L, ws, true,
                       GemmIO{T * p.K, T, reinterpret_cast<__half*>(ws + L.y), nullptr, p.n_local}, s));
  MOE_CUDA(cudaEventRecord(ev[3], s));
  MOE_CUDA(launch_combine_half(p, x_dev, reinterpret_cast<const __half*>(ws + L.y),
                          reinterpret_cast<float*>(ws + L.y_s),
                          reinterpret_cast<int32_t*>(ws + L.slot_row),
                          reinterpret_cast<float*>(ws + L.wts),
                          reinterpret_cast<float*>(ws + L.sgate), out_dev, T, s));
  MOE_CUDA(cudaEventRecord(ev[4], s));
  MOE_CUDA(cudaEventSynchronize(ev[4]));
  for (int i = 0; i < 4; ++i) MOE_CUDA(cudaEventElapsedTime(&stage_ms[i], ev[i], ev[i + 1]));
  return MOE_OK;
}

int moe_route(MoePlan* plan, const float* x_dev, int32_t T, int32_t* topk_ids, float* topk_w,
              int32_t* expert_offsets, int32_t* perm, void* workspace, uint64_t workspace_bytes,
              void* stream) {
  int rc = check_call(plan, T, workspace, workspace_bytes);
  if (rc != MOE_OK || T == 0) return rc;
  if (!x_dev) return fail(MOE_ERR_INVALID, "null x");
  if (misaligned16(x_dev)) return fail(MOE_ERR_INVALID, "x must be 16-byte aligned");
  Plan& p = plan->p;
  if (p.E == 0) return fail(MOE_ERR_UNSUPPORTED, "a dense MLP plan has no routing");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const WsLayout L = ws_layout(p, T);
  char* ws = static_cast<char*>(workspace);
  rc = route_impl(p, L, ws, x_dev, T, false, s);
  if (rc != MOE_OK) return rc;
  const size_t R = static_cast<size_t>(T) * p.K;
  if (topk_ids) MOE_CUDA(cudaMemcpyAsync(topk_ids, ws + L.ids, R * 4, cudaMemcpyDeviceToDevice, s));
  if (topk_w) MOE_CUDA(cudaMemcpyAsync(topk_w, ws + L.wts, R * 4, cudaMemcpyDeviceToDevice, s));
  if (expert_offsets)
    MOE_CUDA(cudaMemcpyAsync(expert_offsets, ws + L.offsets, (p.E + 1) * 4, cudaMemcpyDeviceToDevice, s));
  if (perm) MOE_CUDA(cudaMemcpyAsync(perm, ws + L.perm, R * 4, cudaMemcpyDeviceToDevice, s));
  return MOE_OK;
}

int moe_status(MoePlan* plan, void* stream) {
  if (!plan) return fail(MOE_ERR_INVALID, "null plan");
  Plan& p = plan->p;
  MOE_CUDA(cudaSetDevice(p.device));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int h = 0;
  MOE_CUDA(cudaMemcpyAsync(&h, p.d_err, sizeof(int), cudaMemcpyDeviceToHost, s));
  MOE_CUDA(cudaMemsetAsync(p.d_err, 0, sizeof(int), s));
  MOE_CUDA(cudaStreamSynchronize(s));
  if (h == DEV_OK) return MOE_OK;
  if ((h >= DEV_TIMEOUT_FULL && h <= DEV_TIMEOUT_CONV) || h == DEV_TIMEOUT_PEER)
    return fail(MOE_ERR_TIMEOUT, "a device-side wait ran out of time (code " + std::to_string(h) + ")");
  if (h == DEV_RANGE)
    return fail(MOE_ERR_RANGE, "an activation or expert output overflowed f16 (|v| > 65504)");
  return fail(MOE_ERR_DEVICE, "a kernel reported device error code " + std::to_string(h));
}

int moe_wait_probe(MoePlan* plan, int64_t limit_cycles, void* stream) {
  if (!plan) return fail(MOE_ERR_INVALID, "null plan");
  if (limit_cycles <= 0 || limit_cycles > kWaitLimitCycles)
    return fail(MOE_ERR_INVALID, "limit_cycles must be in (0, 2e9]");
  MOE_CUDA(cudaSetDevice(plan->p.device));
  wait_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(plan->p.d_err, limit_cycles);
  MOE_CUDA(cudaGetLastError());
  return MOE_OK;
}

// ------------------------------------------------------------ expert parallel
static int check_ep(const MoePlan* plan, int32_t n, const void* ws, uint64_t ws_bytes,
                    uint64_t need) {
  if (!plan) return fail(MOE_ERR_INVALID, "null plan");
  if (plan->p.E == 0) return fail(MOE_ERR_UNSUPPORTED, "a dense MLP plan has no experts to exchange");
  if (!plan->p.bound) return fail(MOE_ERR_NOT_BOUND, "moe_bind_layer has not been called");
  if (n < 0) return fail(MOE_ERR_INVALID, "negative row count");
  if (n == 0) return MOE_OK;
  if (!ws || (reinterpret_cast<uintptr_t>(ws) & 255))
    return fail(MOE_ERR_WORKSPACE, "workspace must be a 256-byte aligned device pointer");
  if (ws_bytes < need) return fail(MOE_ERR_WORKSPACE, "workspace too small");
  return MOE_OK;
}

int moe_ep_dispatch(MoePlan* plan, const float* x_dev, int32_t T, void* send_rows,
                    int32_t* send_experts, int32_t* send_offsets, void* workspace,
                    uint64_t workspace_bytes, void* stream) {
  if (!plan) return fail(MOE_ERR_INVALID, "null plan");
  Plan& p = plan->p;
  if (T > p.cfg.max_tokens) return fail(MOE_ERR_INVALID, "T above max_tokens");
  int rc = check_ep(plan, T, workspace, workspace_bytes, T > 0 ? ws_layout(p, T).total : 0);
  if (rc != MOE_OK) return rc;
  if (!send_offsets) return fail(MOE_ERR_INVALID, "null send_offsets");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (T == 0) {
    MOE_CUDA(cudaMemsetAsync(send_offsets, 0, sizeof(int32_t) * (p.E / p.n_local + 1), s));
    return MOE_OK;
  }
  if (!x_dev || !send_rows || !send_experts) return fail(MOE_ERR_INVALID, "null argument");
  if (misaligned16(x_dev)) return fail(MOE_ERR_INVALID, "x must be 16-byte aligned");
  const WsLayout L = ws_layout(p, T);
  char* ws = static_cast<char*>(workspace);
  MOE_CUDA(launch_route(p, L, ws, x_dev, T, true, s, static_cast<__half*>(send_rows)));
  MOE_CUDA(launch_ep_meta(p, reinterpret_cast<int32_t*>(ws + L.perm),
                          reinterpret_cast<int32_t*>(ws + L.ids),
                          reinterpret_cast<int32_t*>(ws + L.offsets), T * p.K, send_experts,
                          send_offsets, s));
  return MOE_OK;
}

uint64_t moe_ep_workspace_bytes(const MoePlan* plan, int32_t R) {
  if (!plan || R <= 0) return 0;
  return ws_layout_ep_experts(plan->p, R, R).total;
}

int moe_ep_experts(MoePlan* plan, const void* recv_rows, const int32_t* recv_experts, int32_t R,
                   void* y_out, void* workspace, uint64_t workspace_bytes, void* stream) {
  if (!plan) return fail(MOE_ERR_INVALID, "null plan");
  Plan& p = plan->p;
  int rc = check_ep(plan, R, workspace, workspace_bytes,
                    R > 0 ? ws_layout_ep_experts(p, R, R).total : 0);
  if (rc != MOE_OK || R == 0) return rc;
  if (!recv_rows || !recv_experts || !y_out) return fail(MOE_ERR_INVALID, "null argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const WsLayout L = ws_layout_ep_experts(p, R, R);
  char* ws = static_cast<char*>(workspace);
  MOE_CUDA(launch_group_rows(p, L, ws, RowKeys{recv_experts, 1, 1, 0, 0},
                             static_cast<const __half*>(recv_rows), p.H, R, s));
  MOE_CUDA(launch_gemm(p, L, ws, false, GemmIO{R, 0, nullptr, nullptr, p.n_local}, s));
  MOE_CUDA(launch_gemm(p, L, ws, true,
                       GemmIO{R, 0, static_cast<__half*>(y_out),
                              reinterpret_cast<const int32_t*>(ws + L.perm), p.n_local},
                       s));
  return MOE_OK;
}

int32_t moe_ep_capacity(const MoePlan* plan, int32_t T) {
  if (!plan || T <= 0 || plan->p.E == 0) return 0;
  const int64_t c = static_cast<int64_t>(T) * std::min(plan->p.K, plan->p.n_local);
  return c > INT32_MAX ? 0 : static_cast<int32_t>(c);
}

// Rows a fixed-capacity exchange moves per rank: world * cap, or 0 if that
// overflows an int32 row count.
static int64_t padded_rows(const Plan& p, int32_t cap) {
  return static_cast<int64_t>(p.E / std::max(p.n_local, 1)) * cap;
}

int moe_ep_dispatch_padded(MoePlan* plan, const float* x_dev, int32_t T, int32_t cap,
                           void* send_rows, void* workspace, uint64_t workspace_bytes,
                           void* stream) {
  if (!plan) return fail(MOE_ERR_INVALID, "null plan");
  Plan& p = plan->p;
  if (T > p.cfg.max_tokens) return fail(MOE_ERR_INVALID, "T above max_tokens");
  int rc = check_ep(plan, T, workspace, workspace_bytes, T > 0 ? ws_layout(p, T).total : 0);
  if (rc != MOE_OK) return rc;
  if (cap <= 0 || cap < moe_ep_capacity(plan, T) || padded_rows(p, cap) > INT32_MAX)
    return fail(MOE_ERR_INVALID, "cap below moe_ep_capacity(plan, T) or too large");
  if (!send_rows || (T > 0 && !x_dev)) return fail(MOE_ERR_INVALID, "null argument");
  if (misaligned16(send_rows) || (T > 0 && misaligned16(x_dev)))
    return fail(MOE_ERR_INVALID, "x and send_rows must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  WsLayout L{};
  if (T > 0) {
    L = ws_layout(p, T);
    MOE_CUDA(launch_route(p, L, ws, x_dev, T, false, s, nullptr));
  }
  MOE_CUDA(launch_ep_pack(p, L, ws, x_dev, T, cap, static_cast<__half*>(send_rows), s));
  return MOE_OK;
}

uint64_t moe_ep_padded_workspace_bytes(const MoePlan* plan, int32_t cap) {
  if (!plan || cap <= 0 || plan->p.E == 0) return 0;
  const int64_t R = padded_rows(plan->p, cap);
  if (R > INT32_MAX) return 0;
  return ws_layout_ep_experts(plan->p, static_cast<int>(R), cap).total;
}

int moe_ep_experts_padded(MoePlan* plan, const void* recv_rows, int32_t cap, void* y_out,
                          void* workspace, uint64_t workspace_bytes, void* stream) {
  if (!plan) return fail(MOE_ERR_INVALID, "null plan");
  Plan& p = plan->p;
  if (cap < 0 || padded_rows(p, cap) > INT32_MAX) return fail(MOE_ERR_INVALID, "bad cap");
  const int R = static_cast<int>(padded_rows(p, cap));
  int rc = check_ep(plan, R, workspace, workspace_bytes,
                    R > 0 ? ws_layout_ep_experts(p, R, cap).total : 0);
  if (rc != MOE_OK || R == 0) return rc;
  if (!recv_rows || !y_out) return fail(MOE_ERR_INVALID, "null argument");
  if (misaligned16(recv_rows)) return fail(MOE_ERR_INVALID, "recv_rows must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const WsLayout L = ws_layout_ep_experts(p, R, cap);
  char* ws = static_cast<char*>(workspace);
  const __half* rows = static_cast<const __half*>(recv_rows);
  // the local expert id is the first int32 of each row's 16-byte tail
  const int32_t* keys = reinterpret_cast<const int32_t*>(rows + p.H);
  MOE_CUDA(launch_group_rows(p, L, ws, RowKeys{keys, (p.H + 8) / 2, 1, 0, 1}, rows, p.H + 8, R, s));
  MOE_CUDA(launch_gemm(p, L, ws, false, GemmIO{R, 0, nullptr, nullptr, p.n_local}, s));
  MOE_CUDA(launch_gemm(p, L, ws, true,
                       GemmIO{R, 0, static_cast<__half*>(y_out),
                              reinterpret_cast<const int32_t*>(ws + L.perm), p.n_local},
                       s));
  return MOE_OK;
}

int32_t moe_ep_token_row_halves(const MoePlan* plan) {
  if (!plan || plan->p.E == 0) return 0;
  return ep_token_row_halves(plan->p);
}

int moe_ep_token_pack(MoePlan* plan, const float* x_dev, int32_t T, int32_t cap, void* send_rows,
                      void* workspace, uint64_t workspace_bytes, void* stream) {
  if (!plan) return fail(MOE_ERR_INVALID, "null plan");
  Plan& p = plan->p;
  if (T > p.cfg.max_tokens) return fail(MOE_ERR_INVALID, "T above max_tokens");
  int rc = check_ep(plan, T, workspace, workspace_bytes, T > 0 ? ws_layout(p, T).total : 0);
  if (rc != MOE_OK) return rc;
  if (cap <= 0 || cap < T) return fail(MOE_ERR_INVALID, "cap must be positive and at least T");
  if (!send_rows || (T > 0 && !x_dev)) return fail(MOE_ERR_INVALID, "null argument");
  if (misaligned16(send_rows) || (T > 0 && misaligned16(x_dev)))
    return fail(MOE_ERR_INVALID, "x and send_rows must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  WsLayout L{};
  if (T > 0) {
    L = ws_layout(p, T);
    MOE_CUDA(launch_route(p, L, ws, x_dev, T, false, s, nullptr));
  }
  MOE_CUDA(launch_ep_token_pack(p, L, ws, x_dev, T, cap, static_cast<__half*>(send_rows), s));
  return MOE_OK;
}

uint64_t moe_ep_gathered_workspace_bytes(const MoePlan* plan, int32_t rows) {
  if (!plan || rows <= 0 || plan->p.E == 0) return 0;
  if (static_cast<int64_t>(rows) * plan->p.K > INT32_MAX) return 0;
  return ws_layout_ep_gathered(plan->p, rows).total;
}

int moe_ep_experts_gathered(MoePlan* plan, const void* recv_rows, int32_t rows, float* partial_out,
                            void* workspace, uint64_t workspace_bytes, void* stream) {
  if (!plan) return fail(MOE_ERR_INVALID, "null plan");
  Plan& p = plan->p;
  if (rows < 0 || static_cast<int64_t>(rows) * p.K > INT32_MAX)
    return fail(MOE_ERR_INVALID, "bad row count");
  int rc = check_ep(plan, rows, workspace, workspace_bytes,
                    rows > 0 ? ws_layout_ep_gathered(p, rows).total : 0);
  if (rc != MOE_OK || rows == 0) return rc;
  if (!recv_rows || !partial_out) return fail(MOE_ERR_INVALID, "null argument");
  if (misaligned16(recv_rows) || misaligned16(partial_out))
    return fail(MOE_ERR_INVALID, "recv_rows and partial_out must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const WsLayout L = ws_layout_ep_gathered(p, rows);
  char* ws = static_cast<char*>(workspace);
  const __half* rec = static_cast<const __half*>(recv_rows);
  const int ld = ep_token_row_halves(p);
  // the K global expert ids follow each record's H values; keys outside this
  // rank's range belong to other ranks and are skipped
  const RowKeys keys{reinterpret_cast<const int32_t*>(rec + p.H), ld / 2, p.K, p.e_begin, 2};
  MOE_CUDA(launch_group_rows(p, L, ws, keys, rec, ld, rows, s));
  const int slots = rows * p.K;
  __half* y = reinterpret_cast<__half*>(ws + L.y);
  MOE_CUDA(launch_gemm(p, L, ws, false, GemmIO{slots, 0, nullptr, nullptr, p.n_local}, s));
  MOE_CUDA(launch_gemm(p, L, ws, true, GemmIO{slots, 0, y, nullptr, p.n_local}, s));
  MOE_CUDA(launch_ep_partial(p, rec, rows, y, reinterpret_cast<const int32_t*>(ws + L.slot_row),
                             partial_out, s));
  return MOE_OK;
}

int moe_ep_combine_partial(MoePlan* plan, const float* x_dev, int32_t T, const float* partial,
                           float* out_dev, void* workspace, uint64_t workspace_bytes, void* stream) {
  if (!plan) return fail(MOE_ERR_INVALID, "null plan");
  Plan& p = plan->p;
  int rc = check_ep(plan, T, workspace, workspace_bytes, T > 0 ? ws_layout(p, T).total : 0);
  if (rc != MOE_OK || T == 0) return rc;
  if (!x_dev || !partial || !out_dev) return fail(MOE_ERR_INVALID, "null argument");
  if (x_dev == out_dev) return fail(MOE_ERR_INVALID, "x and out may not alias");
  if (misaligned16(x_dev) || misaligned16(partial) || misaligned16(out_dev))
    return fail(MOE_ERR_INVALID, "x, partial and out must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const WsLayout L = ws_layout(p, T);
  char* ws = static_cast<char*>(workspace);
  MOE_CUDA(launch_combine_partial(p, x_dev, partial, reinterpret_cast<float*>(ws + L.y_s),
                                  reinterpret_cast<float*>(ws + L.sgate), out_dev, T, s));
  return MOE_OK;
}

// ------------------------------------------------------------ exchange over peer memory
static int p2p_peers(const MoePlan* plan, int32_t rank, int32_t world, void* const* recv,
                     float* const* part, int32_t* const* flags, P2PPeers* out) {
  if (world < 1 || world > kMaxP2PRanks || rank < 0 || rank >= world)
    return fail(MOE_ERR_INVALID, "rank / world outside [0, 8)");
  if (plan->p.E / std::max(plan->p.n_local, 1) != world)
    return fail(MOE_ERR_INVALID, "world does not match the plan's expert share");
  if (plan->p.e_begin != rank * plan->p.n_local)
    return fail(MOE_ERR_INVALID, "rank does not match the plan's expert range");
  *out = P2PPeers{};
  for (int d = 0; d < world; ++d) {
    if ((recv && !recv[d]) || (part && !part[d]) || !flags || !flags[d])
      return fail(MOE_ERR_INVALID, "null peer buffer");
    if (recv) out->recv[d] = recv[d];
    if (part) out->part[d] = part[d];
    out->flags[d] = flags[d];
  }
  return MOE_OK;
}

int moe_ep_p2p_pack(MoePlan* plan, const float* x_dev, int32_t T, int32_t cap, int32_t rank,
                    int32_t world, void* const* peer_recv, int32_t* const* peer_flags, int32_t epoch,
                    int32_t* done, void* workspace, uint64_t workspace_bytes, void* stream) {
  if (!plan) return fail(MOE_ERR_INVALID, "null plan");
  Plan& p = plan->p;
  if (T > p.cfg.max_tokens) return fail(MOE_ERR_INVALID, "T above max_tokens");
  int rc = check_ep(plan, T, workspace, workspace_bytes, T > 0 ? ws_layout(p, T).total : 0);
  if (rc != MOE_OK) return rc;
  if (cap <= 0 || cap < T) return fail(MOE_ERR_INVALID, "cap must be positive and at least T");
  if (epoch <= 0) return fail(MOE_ERR_INVALID, "epoch must be positive");
  if (!done || !peer_recv || (T > 0 && !x_dev)) return fail(MOE_ERR_INVALID, "null argument");
  P2PPeers peers;
  rc = p2p_peers(plan, rank, world, peer_recv, nullptr, peer_flags, &peers);
  if (rc != MOE_OK) return rc;
  for (int d = 0; d < world; ++d)
    if (misaligned16(peer_recv[d])) return fail(MOE_ERR_INVALID, "receive buffers must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  WsLayout L{};
  if (T > 0) {
    L = ws_layout(p, T);
    MOE_CUDA(launch_route(p, L, ws, x_dev, T, false, s, nullptr));
  }
  MOE_CUDA(launch_p2p_pack(p, L, ws, x_dev, T, cap, rank, world, peers, epoch, done, s));
  return MOE_OK;
}

int moe_ep_p2p_wait(MoePlan* plan, const int32_t* flags, int32_t world, int32_t epoch,
                    int64_t limit_cycles, void* stream) {
  if (!plan) return fail(MOE_ERR_INVALID, "null plan");
  if (!flags || world < 1 || world > kMaxP2PRanks || epoch <= 0)
    return fail(MOE_ERR_INVALID, "bad flags / world / epoch");
  if (limit_cycles <= 0 || limit_cycles > kWaitLimitCycles)
    return fail(MOE_ERR_INVALID, "limit_cycles must be in (0, 2e9]");
  MOE_CUDA(launch_p2p_wait(flags, world, epoch, limit_cycles, plan->p.d_err,
                           static_cast<cudaStream_t>(stream)));
  return MOE_OK;
}

int moe_ep_p2p_experts(MoePlan* plan, const void* recv_rows, int32_t cap, int32_t rank,
                       int32_t world, float* const* peer_part, int32_t* const* peer_flags,
                       int32_t epoch, int32_t* done, void* workspace, uint64_t workspace_bytes,
                       void* stream) {
  if (!plan) return fail(MOE_ERR_INVALID, "null plan");
  Plan& p = plan->p;
  if (cap <= 0 || static_cast<int64_t>(cap) * world * p.K > INT32_MAX)
    return fail(MOE_ERR_INVALID, "bad cap");
  const int rows = cap * world;
  int rc = check_ep(plan, rows, workspace, workspace_bytes, ws_layout_ep_gathered(p, rows).total);
  if (rc != MOE_OK) return rc;
  if (!recv_rows || !done || !peer_part || epoch <= 0) return fail(MOE_ERR_INVALID, "null argument");
  if (misaligned16(recv_rows)) return fail(MOE_ERR_INVALID, "recv_rows must be 16-byte aligned");
  P2PPeers peers;
  rc = p2p_peers(plan, rank, world, nullptr, peer_part, peer_flags, &peers);
  if (rc != MOE_OK) return rc;
  for (int d = 0; d < world; ++d)
    if (misaligned16(peer_part[d])) return fail(MOE_ERR_INVALID, "partial buffers must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const WsLayout L = ws_layout_ep_gathered(p, rows);
  char* ws = static_cast<char*>(workspace);
  const __half* rec = static_cast<const __half*>(recv_rows);
  const int ld = ep_token_row_halves(p);
  const RowKeys keys{reinterpret_cast<const int32_t*>(rec + p.H), ld / 2, p.K, p.e_begin, 2};
  MOE_CUDA(launch_group_rows(p, L, ws, keys, rec, ld, rows, s));
  const int slots = rows * p.K;
  __half* y = reinterpret_cast<__half*>(ws + L.y);
  MOE_CUDA(launch_gemm(p, L, ws, false, GemmIO{slots, 0, nullptr, nullptr, p.n_local}, s));
  MOE_CUDA(launch_gemm(p, L, ws, true, GemmIO{slots, 0, y, nullptr, p.n_local}, s));
  MOE_CUDA(launch_p2p_partial(p, rec, cap, y, reinterpret_cast<const int32_t*>(ws + L.slot_row), rank,
                              world, peers, epoch, done, s));
  return MOE_OK;
}

int moe_ep_p2p_combine(MoePlan* plan, const float* x_dev, int32_t T, const float* part,
                       int32_t cap, int32_t world, float* out_dev, void* workspace,
                       uint64_t workspace_bytes, void* stream) {
  if (!plan) return fail(MOE_ERR_INVALID, "null plan");
  Plan& p = plan->p;
  int rc = check_ep(plan, T, workspace, workspace_bytes, T > 0 ? ws_layout(p, T).total : 0);
  if (rc != MOE_OK || T == 0) return rc;
  if (!x_dev || !part || !out_dev) return fail(MOE_ERR_INVALID, "null argument");
  if (cap < T || world < 1 || world > kMaxP2PRanks) return fail(MOE_ERR_INVALID, "bad cap / world");
  if (x_dev == out_dev) return fail(MOE_ERR_INVALID, "x and out may not alias");
  if (misaligned16(x_dev) || misaligned16(part) || misaligned16(out_dev))
    return fail(MOE_ERR_INVALID, "x, part and out must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const WsLayout L = ws_layout(p, T);
  char* ws = static_cast<char*>(workspace);
  MOE_CUDA(launch_p2p_combine(p, x_dev, part, cap, world, reinterpret_cast<float*>(ws + L.y_s),
                              reinterpret_cast<float*>(ws + L.sgate), out_dev, T, s));
  return MOE_OK;
}

int moe_ep_shared(MoePlan* plan, int32_t T, void* workspace, uint64_t workspace_bytes,
                  void* stream) {
  if (!plan) return fail(MOE_ERR_INVALID, "null plan");
  Plan& p = plan->p;
  int rc = check_ep(plan, T, workspace, workspace_bytes, T > 0 ? ws_layout(p, T).total : 0);
  if (rc != MOE_OK || T == 0 || p.SI == 0) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const WsLayout L = ws_layout(p, T);
  char* ws = static_cast<char*>(workspace);
  MOE_CUDA(launch_shared_tiles(p, L, ws, T, s));
  MOE_CUDA(launch_gemm(p, L, ws, false, GemmIO{T * p.K, T, nullptr, nullptr, 0}, s));
  MOE_CUDA(launch_gemm(p, L, ws, true, GemmIO{T * p.K, T, nullptr, nullptr, 0}, s));
  return MOE_OK;
}

int moe_ep_combine(MoePlan* plan, const float* x_dev, int32_t T, const void* y_back,
                   float* out_dev, void* workspace, uint64_t workspace_bytes, void* stream) {
  if (!plan) return fail(MOE_ERR_INVALID, "null plan");
  Plan& p = plan->p;
  int rc = check_ep(plan, T, workspace, workspace_bytes, T > 0 ? ws_layout(p, T).total : 0);
  if (rc != MOE_OK || T == 0) return rc;
  if (!x_dev || !y_back || !out_dev) return fail(MOE_ERR_INVALID, "null argument");
  if (x_dev == out_dev) return fail(MOE_ERR_INVALID, "x and out may not alias");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const WsLayout L = ws_layout(p, T);
  char* ws = static_cast<char*>(workspace);
  MOE_CUDA(launch_combine_half(p, x_dev, static_cast<const __half*>(y_back),
                               reinterpret_cast<float*>(ws + L.y_s),
                               reinterpret_cast<int32_t*>(ws + L.slot_row),
                               reinterpret_cast<float*>(ws + L.wts),
                               reinterpret_cast<float*>(ws + L.sgate), out_dev, T, s));
  return MOE_OK;
}

// ------------------------------------------------------------ runtime wrappers
int moe_rt_device_count(int32_t* count) {
  int n = 0;
  MOE_CUDA(cudaGetDeviceCount(&n));
  if (count) *count = n;
  return MOE_OK;
}
int moe_rt_set_device(int32_t device) {
  MOE_CUDA(cudaSetDevice(device));
  return MOE_OK;
}
int moe_rt_can_access_peer(int32_t device, int32_t peer, int32_t* can_access) {
  if (!can_access) return fail(MOE_ERR_INVALID, "null out pointer");
  int ok = 0;
  MOE_CUDA(cudaDeviceCanAccessPeer(&ok, device, peer));
  *can_access = ok;
  return MOE_OK;
}
int moe_rt_malloc(uint64_t nbytes, void** dev_ptr) {
  if (!dev_ptr) return fail(MOE_ERR_INVALID, "null out pointer");
  MOE_CUDA(cudaMalloc(dev_ptr, nbytes));
  return MOE_OK;
}
static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handles are 64 bytes in the C ABI");

int moe_rt_ipc_get_handle(const void* dev_ptr, void* handle) {
  if (!dev_ptr || !handle) return fail(MOE_ERR_INVALID, "null argument");
  cudaIpcMemHandle_t h;
  MOE_CUDA(cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr)));
  std::memcpy(handle, &h, sizeof(h));
  return MOE_OK;
}

int moe_rt_ipc_open_handle(const void* handle, void** dev_ptr) {
  if (!handle || !dev_ptr) return fail(MOE_ERR_INVALID, "null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  MOE_CUDA(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return MOE_OK;
}

int moe_rt_ipc_close_handle(void* dev_ptr) {
  if (!dev_ptr) return fail(MOE_ERR_INVALID, "null argument");
  MOE_CUDA(cudaIpcCloseMemHandle(dev_ptr));
  return MOE_OK;
}

int moe_rt_free(void* dev_ptr) {
  MOE_CUDA(cudaFree(dev_ptr));
  return MOE_OK;
}
int moe_rt_malloc_host(uint64_t nbytes, void** host_ptr) {
  if (!host_ptr) return fail(MOE_ERR_INVALID, "null out pointer");
  MOE_CUDA(cudaMallocHost(host_ptr, nbytes));
  return MOE_OK;
}
int moe_rt_free_host(void* host_ptr) {
  MOE_CUDA(cudaFreeHost(host_ptr));
  return MOE_OK;
}
int moe_rt_stream_create(void** stream) {
  if (!stream) return fail(MOE_ERR_INVALID, "null out pointer");
  cudaStream_t s;
  MOE_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  *stream = s;
  return MOE_OK;
}
int moe_rt_stream_destroy(void* stream) {
  MOE_CUDA(cudaStreamDestroy(static_cast<cudaStream_t>(stream)));
  return MOE_OK;
}
int moe_rt_memcpy_h2d_async(void* dst_dev, const void* src_host, uint64_t nbytes, void* stream) {
  MOE_CUDA(cudaMemcpyAsync(dst_dev, src_host, nbytes, cudaMemcpyHostToDevice,
                           static_cast<cudaStream_t>(stream)));
  return MOE_OK;
}
int moe_rt_memcpy_d2h_async(void* dst_host, const void* src_dev, uint64_t nbytes, void* stream) {
  MOE_CUDA(cudaMemcpyAsync(dst_host, src_dev, nbytes, cudaMemcpyDeviceToHost,
                           static_cast<cudaStream_t>(stream)));
  return MOE_OK;
}
int moe_rt_memcpy_d2d_async(void* dst_dev, const void* src_dev, uint64_t nbytes, void* stream) {
  MOE_CUDA(cudaMemcpyAsync(dst_dev, src_dev, nbytes, cudaMemcpyDeviceToDevice,
                           static_cast<cudaStream_t>(stream)));
  return MOE_OK;
}
int moe_rt_event_record(void* stream, void** event) {
  if (!event) return fail(MOE_ERR_INVALID, "null out pointer");
  cudaEvent_t e;
  MOE_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  MOE_CUDA(cudaEventRecord(e, static_cast<cudaStream_t>(stream)));
  *event = e;
  return MOE_OK;
}
int moe_rt_event_destroy(void* event) {
  MOE_CUDA(cudaEventDestroy(static_cast<cudaEvent_t>(event)));
  return MOE_OK;
}
int moe_rt_stream_wait_event(void* stream, void* event) {
  MOE_CUDA(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), static_cast<cudaEvent_t>(event), 0));
  return MOE_OK;
}
int moe_rt_stream_synchronize(void* stream) {
  MOE_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  return MOE_OK;
}

}  // extern "C"
