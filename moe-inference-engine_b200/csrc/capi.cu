// extern "C" entry points of libmie.so (declared in include/mie.h): argument
// validation, launch geometry, and the decode-step launch sequence.
#include <cstdio>
#include <cstring>

#include "kernels.h"

namespace mie {

namespace {
thread_local char g_last_error[256] = "";
}

void note_cuda_error(cudaError_t e, const char* what) {
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%d)", what, cudaGetErrorString(e), (int)e);
}

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
int esize(int dtype) { return dtype == MIE_BF16 ? 2 : 4; }
bool dtype_ok(int d) { return d == MIE_F32 || d == MIE_BF16; }
bool rows16(int elems, int dtype) { return ((int64_t)elems * esize(dtype)) % 16 == 0; }

constexpr int kMaxRowElems = 16 * 1024;  // longest weight row (elements) the kernels accept

int check_moe(const mie_moe_args& a, bool route_only) {
  if (!dtype_ok(a.dtype) || !dtype_ok(a.x_dtype) || (!route_only && !dtype_ok(a.out_dtype))) return MIE_ERR_UNSUPPORTED;
  if (a.top_k != 2 || a.num_experts < 2 || a.num_experts > 32) return MIE_ERR_UNSUPPORTED;
  if (a.hidden_dim <= 0 || a.expert_hidden_dim <= 0) return MIE_ERR_INVALID;
  if (!rows16(a.hidden_dim, a.dtype) || !rows16(a.expert_hidden_dim, a.dtype)) return MIE_ERR_UNSUPPORTED;
  if (a.expert_hidden_dim > kMaxRowElems || a.hidden_dim > kMaxRowElems) return MIE_ERR_UNSUPPORTED;
  if (!a.x || !a.router_w || !aligned16(a.router_w)) return MIE_ERR_INVALID;
  if (a.norm != MIE_NORM_NONE && !a.norm_w) return MIE_ERR_INVALID;
  if (route_only) return MIE_OK;
  if (a.act != MIE_ACT_GELU && a.act != MIE_ACT_SWIGLU) return MIE_ERR_UNSUPPORTED;
  if (a.expert_bits != 0) {
    // quantized experts: int8 / int4 rows of whole 16-byte pieces and groups
    if (a.expert_bits != 8 && a.expert_bits != 4) return MIE_ERR_UNSUPPORTED;
    const int g = a.group_size;
    if (g < 32 || (g & (g - 1)) || a.hidden_dim % g || a.expert_hidden_dim % g) return MIE_ERR_UNSUPPORTED;
    if (((int64_t)a.hidden_dim * a.expert_bits / 8) % 16 || ((int64_t)a.expert_hidden_dim * a.expert_bits / 8) % 16)
      return MIE_ERR_UNSUPPORTED;
    if (!a.w1_scale || !a.w2_scale || (a.act == MIE_ACT_SWIGLU && !a.w3_scale)) return MIE_ERR_INVALID;
  }
  if (!a.w1 || !a.w2 || !aligned16(a.w1) || !aligned16(a.w2)) return MIE_ERR_INVALID;
  if (a.act == MIE_ACT_SWIGLU && (!a.w3 || !aligned16(a.w3))) return MIE_ERR_INVALID;
  if (!a.hidden || !a.out || !a.sync) return MIE_ERR_INVALID;
  if (a.expert_count < 0 || a.expert_base < 0 || a.expert_base + a.expert_count > a.num_experts)
    return MIE_ERR_INVALID;
  if (a.peer_world > 1) {
    // the fused expert-parallel all-reduce (one word per row per rank)
    if (a.peer_world > MIE_PEER_MAX_RANKS || a.peer_rank < 0 || a.peer_rank >= a.peer_world || !a.peer_seq)
      return MIE_ERR_INVALID;
    for (int r = 0; r < a.peer_world; ++r)
      if (!a.peer_bufs[r] || (reinterpret_cast<uintptr_t>(a.peer_bufs[r]) & 7u)) return MIE_ERR_INVALID;
  }
  return MIE_OK;
}

int run_moe(const mie_moe_args& a, cudaStream_t st, bool pdl, bool route_only) {
  const int rc = check_moe(a, route_only);
  if (rc) return rc;
  int grid = a.grid > 0 ? a.grid : num_sms();
  if (grid > num_sms()) grid = num_sms();  // grid barrier: all CTAs co-resident
  if (route_only) grid = 1;
  MoeLayout L = moe_layout(a, grid, 0, 0);
  L.route_only = route_only ? 1 : 0;
  if (L.smem > (uint32_t)kMaxDynSmem) return MIE_ERR_UNSUPPORTED;
  if (a.expert_bits != 0 && !route_only) return moe_decode_q_launch(a, L, grid, st, pdl);
  return moe_decode_launch(a, L, grid, st, pdl);
}

// with_scratch false: the request is checked without its partials / counters /
// max_splits (the fixed-scratch entry point supplies those itself).
int check_attn(const mie_attn_args& a, bool with_scratch = true) {
  if (!dtype_ok(a.kv_dtype) || !dtype_ok(a.q_dtype) || !dtype_ok(a.out_dtype)) return MIE_ERR_UNSUPPORTED;
  switch (a.head_dim) {
    case 4: case 8: case 16: case 32: case 64: case 96: case 128: break;
    default: return MIE_ERR_UNSUPPORTED;
  }
  if (a.num_heads <= 0 || a.block_size <= 0 || a.splits <= 0) return MIE_ERR_INVALID;
  if (with_scratch && a.splits > a.max_splits) return MIE_ERR_INVALID;
  if (!a.q || !a.k || !a.v || !a.out) return MIE_ERR_INVALID;
  if (with_scratch && a.splits > 1 && (!a.partials || !a.counters)) return MIE_ERR_INVALID;
  if (!a.ctx_dev && (a.ctx_len < 1 || a.ctx_len > a.max_ctx)) return MIE_ERR_INVALID;
  if (a.stride_tok != a.head_dim) return MIE_ERR_UNSUPPORTED;
  if (rows16(a.head_dim, a.kv_dtype)) {
    const int64_t e = esize(a.kv_dtype);
    if (!aligned16(a.k) || !aligned16(a.v) || (a.stride_block * e) % 16 || (a.stride_head * e) % 16)
      return MIE_ERR_INVALID;
  }
  return MIE_OK;
}

int run_attn(const mie_attn_args& a, cudaStream_t st, bool pdl) {
  const int rc = check_attn(a);
  if (rc) return rc;
  AttnLayout L = attn_layout(a);
  if (L.smem > (uint32_t)kMaxDynSmem) return MIE_ERR_UNSUPPORTED;
  return attn_decode_launch(a, L, st, pdl);
}

int check_qkv(const mie_qkv_args& a) {
  if (!dtype_ok(a.dtype) || !dtype_ok(a.kv_dtype)) return MIE_ERR_UNSUPPORTED;
  if (a.num_heads <= 0 || a.head_dim <= 0 || a.head_dim % 2 || a.num_heads * a.head_dim != a.hidden_dim)
    return MIE_ERR_INVALID;
  if (!rows16(a.hidden_dim, a.dtype) || a.hidden_dim > kMaxRowElems) return MIE_ERR_UNSUPPORTED;
  if (!a.x || !a.w || !aligned16(a.w) || !a.pos || !a.q_out || !a.k_cache || !a.v_cache) return MIE_ERR_INVALID;
  if (a.embedding && !a.token) return MIE_ERR_INVALID;
  if (a.norm != MIE_NORM_NONE && !a.norm_w) return MIE_ERR_INVALID;
  if ((a.rope_cos == nullptr) != (a.rope_sin == nullptr)) return MIE_ERR_INVALID;
  if (a.block_size <= 0) return MIE_ERR_INVALID;
  return MIE_OK;
}

int run_qkv(const mie_qkv_args& a, cudaStream_t st, bool pdl) {
  const int rc = check_qkv(a);
  if (rc) return rc;
  const int U = 3 * a.num_heads * (a.head_dim / 2);
  int grid = a.grid > 0 ? a.grid : num_sms();
  if (grid > U) grid = U;
  GemvLayout L = qkv_layout(a, grid);
  return qkv_launch(a, L, grid, st, pdl);
}

int run_proj(const mie_proj_args& a, cudaStream_t st, bool pdl) {
  if (!dtype_ok(a.dtype)) return MIE_ERR_UNSUPPORTED;
  if (a.rows <= 0 || a.cols <= 0 || !a.w || !aligned16(a.w) || !a.out) return MIE_ERR_INVALID;
  if (a.attn_partials) {
    if (a.attn_heads <= 0 || a.attn_heads > 64 || a.attn_splits <= 0 || a.attn_splits > 64 ||
        a.attn_splits > a.attn_max_splits || a.attn_heads * a.attn_head_dim != a.cols)
      return MIE_ERR_INVALID;
  } else if (!a.in) {
    return MIE_ERR_INVALID;
  }
  if (!rows16(a.cols, a.dtype) || a.cols > kMaxRowElems) return MIE_ERR_UNSUPPORTED;
  int grid = a.grid > 0 ? a.grid : num_sms();
  if (grid > a.rows) grid = a.rows;
  GemvLayout L = proj_layout(a, grid);
  return proj_launch(a, L, grid, st, pdl);
}

int run_lmhead(const mie_lmhead_args& a, cudaStream_t st, bool pdl) {
  if (!dtype_ok(a.dtype)) return MIE_ERR_UNSUPPORTED;
  if (a.vocab <= 0 || a.hidden_dim <= 0 || !a.x || !a.w || !aligned16(a.w)) return MIE_ERR_INVALID;
  if (!rows16(a.hidden_dim, a.dtype) || a.hidden_dim > kMaxRowElems) return MIE_ERR_UNSUPPORTED;
  if (!a.partial_val || !a.partial_idx || !a.counter) return MIE_ERR_INVALID;
  if (a.norm != MIE_NORM_NONE && !a.norm_w) return MIE_ERR_INVALID;
  int grid = a.grid > 0 ? a.grid : num_sms();
  if (grid > a.vocab) grid = a.vocab;
  GemvLayout L = lmhead_layout(a, grid);
  return lmhead_launch(a, L, grid, st, pdl);
}

// ---- decode step ---------------------------------------------------------

mie_qkv_args step_qkv(const mie_step_desc& d, int l) {
  const mie_layer_desc& ly = d.layers[l];
  mie_qkv_args a = {};
  a.dtype = d.dtype;
  a.kv_dtype = d.kv_dtype;
  a.hidden_dim = d.hidden_dim;
  a.num_heads = d.num_heads;
  a.head_dim = d.head_dim;
  a.norm = d.norm;
  a.eps = d.eps;
  a.norm_w = ly.attn_norm_w;
  a.norm_b = ly.attn_norm_b;
  a.x = d.x;
  a.x_add = (l > 0 && d.moe_partial) ? d.moe_partial : nullptr;
  a.embedding = l == 0 ? d.embedding : nullptr;
  a.pos_embedding = l == 0 ? d.pos_embedding : nullptr;
  a.token = d.token;
  a.vocab = d.vocab;
  a.w = ly.qkv_w;
  a.b = ly.qkv_b;
  a.rope_cos = d.rope_cos;
  a.rope_sin = d.rope_sin;
  a.pos = d.pos;
  a.max_pos = d.max_pos;
  a.q_out = d.q;
  a.k_cache = ly.k_cache;
  a.v_cache = ly.v_cache;
  a.block_table = d.block_table;
  a.num_blocks = d.num_blocks;
  a.block_size = d.block_size;
  a.stride_block = d.kv_stride_block;
  a.stride_head = d.kv_stride_head;
  a.stride_tok = d.kv_stride_tok;
  a.status = d.status;
  a.skip = d.done;
  return a;
}

mie_attn_args step_attn(const mie_step_desc& d, int l) {
  const mie_layer_desc& ly = d.layers[l];
  mie_attn_args a = {};
  a.kv_dtype = d.kv_dtype;
  a.q_dtype = MIE_F32;
  a.out_dtype = MIE_F32;
  a.num_heads = d.num_heads;
  a.head_dim = d.head_dim;
  a.q = d.q;
  a.k = ly.k_cache;
  a.v = ly.v_cache;
  a.block_table = d.block_table;
  a.num_blocks = d.num_blocks;
  a.block_size = d.block_size;
  a.stride_block = d.kv_stride_block;
  a.stride_head = d.kv_stride_head;
  a.stride_tok = d.kv_stride_tok;
  a.ctx_dev = d.pos;
  a.ctx_dev_offset = 1;
  a.max_ctx = d.max_pos;
  a.scale = d.attn_scale;
  a.out = d.attn_out;
  a.partials = d.attn_partials;
  a.counters = d.attn_counters;
  a.splits = d.attn_splits;
  a.max_splits = d.max_splits;
  a.new_token_last = 1;
  a.status = d.status;
  a.skip = d.done;
  a.defer_merge = 1;  // proj_kernel merges the split partials
  return a;
}

mie_proj_args step_proj(const mie_step_desc& d, int l) {
  const mie_layer_desc& ly = d.layers[l];
  mie_proj_args a = {};
  a.dtype = d.dtype;
  a.rows = d.hidden_dim;
  a.cols = d.num_heads * d.head_dim;
  a.w = ly.out_w;
  a.b = ly.out_b;
  a.in = d.attn_out;
  a.attn_partials = d.attn_partials;
  a.attn_heads = d.num_heads;
  a.attn_head_dim = d.head_dim;
  a.attn_splits = d.attn_splits;
  a.attn_max_splits = d.max_splits;
  a.out = d.x;
  a.add = (l > 0 && d.moe_partial) ? d.moe_partial : nullptr;
  a.accumulate = 1;
  a.status = d.status;
  a.skip = d.done;
  return a;
}

mie_moe_args step_moe(const mie_step_desc& d, int l) {
  const mie_layer_desc& ly = d.layers[l];
  mie_moe_args a = {};
  a.dtype = d.dtype;
  a.x_dtype = MIE_F32;
  a.out_dtype = MIE_F32;
  a.hidden_dim = d.hidden_dim;
  a.expert_hidden_dim = d.expert_hidden_dim;
  a.num_experts = d.num_experts;
  a.top_k = d.top_k;
  a.act = d.act;
  a.norm = d.norm;
  a.eps = d.eps;
  a.x = d.x;
  a.norm_w = ly.moe_norm_w;
  a.norm_b = ly.moe_norm_b;
  a.router_w = ly.router_w;
  a.w1 = ly.w1;
  a.b1 = ly.b1;
  a.w3 = ly.w3;
  a.w2 = ly.w2;
  a.b2 = ly.b2;
  a.hidden = d.moe_hidden;
  if (d.moe_partial) {
    a.out = d.moe_partial;
    a.residual = 0;
  } else {
    a.out = d.x;
    a.residual = 1;
  }
  a.sync = d.moe_sync;
  a.status = d.status;
  a.skip = d.done;
  a.expert_base = d.expert_base;
  a.expert_count = d.expert_count;
  if (d.expert_bits) {  // quantized experts: the grouped kernel
    a.expert_bits = d.expert_bits;
    a.group_size = d.group_size;
    a.w1_scale = ly.w1_scale;
    a.w3_scale = ly.w3_scale;
    a.w2_scale = ly.w2_scale;
  }
  if (d.moe_peer) {  // expert parallel: the MoE kernel completes the all-reduce of its partial
    const mie_peer_reduce_args& p = *d.moe_peer;
    a.peer_rank = p.rank;
    a.peer_world = p.world;
    a.peer_seq = p.seq;
    for (int r = 0; r < MIE_PEER_MAX_RANKS; ++r) a.peer_bufs[r] = r < p.world ? p.bufs[r] : nullptr;
    a.peer_wait_limit_ns = p.wait_limit_ns;
  }
  return a;
}

mie_lmhead_args step_lmhead(const mie_step_desc& d) {
  mie_lmhead_args a = {};
  a.dtype = d.dtype;
  a.vocab = d.vocab;
  a.hidden_dim = d.hidden_dim;
  a.norm = d.norm;
  a.eps = d.eps;
  a.norm_w = d.final_norm_w;
  a.norm_b = d.final_norm_b;
  a.x = d.x;
  a.x_add = d.moe_partial;
  a.w = d.embedding;
  a.b = d.lm_bias;
  a.logits = d.logits;
  a.partial_val = d.lm_partial_val;
  a.partial_idx = d.lm_partial_idx;
  a.counter = d.lm_counter;
  a.token_out = d.token;
  a.pos = d.pos;
  a.tokens_log = d.tokens_log;
  a.log_count = d.log_count;
  a.log_capacity = d.log_capacity;
  a.done = d.done;
  a.eos_id = d.eos_id;
  a.status = d.status;
  a.skip = d.done;
  a.grid = d.lm_grid;
  return a;
}

// The persistent kernel that runs a step and its geometry.
struct StepPlan {
  int cluster;  // 1: the cluster step (cg), 0: the one-CTA-per-SM step (g)
  StepGeom g;
  CGeom cg;
  int64_t words() const { return cluster ? cg.words : g.words; }
};

// Persistent step: geometry for this device plus the checks the per-op
// launchers would otherwise make (alignment of every weight row base and of
// the K/V caches, which the kernel copies in 16-byte units).  The cluster
// step runs every step whose shapes it takes, unless d.step_kernel forces
// the one-CTA-per-SM step.
int persistent_geometry(const mie_step_desc& d, StepPlan* plan) {
  if (!d.layers || !d.embedding || !d.token || !d.pos || !d.x || !d.lm_partial_val || !d.lm_partial_idx ||
      !d.lm_counter)
    return MIE_ERR_INVALID;
  if (d.step_kernel < MIE_STEP_AUTO || d.step_kernel > MIE_STEP_CLUSTER) return MIE_ERR_INVALID;
  plan->cluster = 0;
  int rc = MIE_ERR_UNSUPPORTED;
  if (d.step_kernel != MIE_STEP_FLAT) {
    rc = cstep_geometry(d, &plan->cg);
    if (rc == MIE_OK)
      plan->cluster = 1;
    else if (d.step_kernel == MIE_STEP_CLUSTER || (d.moe_peer && d.moe_peer->world > 1))
      return rc;  // expert parallel: no other persistent kernel takes it
  }
  if (!plan->cluster) rc = step_geometry(d, num_sms(), &plan->g);
  if (rc) return rc;
  if (d.norm != MIE_NORM_NONE && !d.final_norm_w) return MIE_ERR_INVALID;
  if ((d.rope_cos == nullptr) != (d.rope_sin == nullptr)) return MIE_ERR_INVALID;
  if (d.block_size <= 0 || d.max_pos <= 0) return MIE_ERR_INVALID;
  if (!aligned16(d.embedding) || (d.final_norm_w && !aligned16(d.final_norm_w)) ||
      (d.final_norm_b && !aligned16(d.final_norm_b)))
    return MIE_ERR_INVALID;
  for (int l = 0; l < d.num_layers; ++l) {
    const mie_layer_desc& y = d.layers[l];
    if (!y.qkv_w || !y.out_w || !y.router_w || !y.w1 || !y.w2 || !y.k_cache || !y.v_cache) return MIE_ERR_INVALID;
    if (d.act == MIE_ACT_SWIGLU && !y.w3) return MIE_ERR_INVALID;
    if (d.norm == MIE_NORM_NONE || !y.attn_norm_w || !y.moe_norm_w) return MIE_ERR_UNSUPPORTED;
    if (!aligned16(y.qkv_w) || !aligned16(y.out_w) || !aligned16(y.router_w) || !aligned16(y.w1) ||
        !aligned16(y.w2) || (y.w3 && !aligned16(y.w3)) || !aligned16(y.k_cache) || !aligned16(y.v_cache) ||
        !aligned16(y.attn_norm_w) || !aligned16(y.moe_norm_w) || (y.attn_norm_b && !aligned16(y.attn_norm_b)) ||
        (y.moe_norm_b && !aligned16(y.moe_norm_b)))
      return MIE_ERR_INVALID;
  }
  return MIE_OK;
}

int check_step(const mie_step_desc& d) {
  if (!d.layers || d.num_layers <= 0 || !d.embedding || !d.token || !d.pos || !d.x || !d.q || !d.attn_out ||
      !d.moe_hidden || !d.moe_sync || !d.lm_partial_val || !d.lm_partial_idx || !d.lm_counter)
    return MIE_ERR_INVALID;
  if (d.attn_splits > 1 && (!d.attn_partials || !d.attn_counters)) return MIE_ERR_INVALID;
  return MIE_OK;
}

}  // namespace
}  // namespace mie

using namespace mie;

extern "C" {

int mie_version(void) { return 1; }

const char* mie_status_string(int code) {
  switch (code) {
    case MIE_OK: return "ok";
    case MIE_ERR_INVALID: return "invalid argument (null pointer, size or alignment)";
    case MIE_ERR_UNSUPPORTED: return "unsupported shape or dtype for the sm_100a kernels";
    case MIE_ERR_CUDA: return "CUDA runtime error";
    case MIE_ERR_TIMEOUT: return "device wait timed out";
    case MIE_ERR_RANGE: return "device index out of range (block id, position, expert or token)";
    case MIE_ERR_SCRATCH_LIMIT:
      return "request exceeds the fixed scratch of mie_attn_decode_fixed_scratch "
             "(num_heads <= 64, num_heads * splits * (head_dim + 2) <= 65536)";
    default: return "unknown status";
  }
}

int mie_num_sms(int device) {
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return -1;
  return n;
}

int mie_init(int device) {
  int cur = 0;
  if (cudaGetDevice(&cur) != cudaSuccess) return MIE_ERR_CUDA;
  if (device >= 0 && device != cur) {
    if (cudaSetDevice(device) != cudaSuccess) return MIE_ERR_CUDA;
  }
  g_last_error[0] = 0;
  moe_set_attributes();
  moe_q_set_attributes();
  attn_set_attributes();
  gemv_set_attributes();
  step_set_attributes();
  cstep_set_attributes();
  gemm_set_attributes();
  (void)num_sms();
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) note_cuda_error(e, "mie_init");
  if (device >= 0 && device != cur) cudaSetDevice(cur);
  return (e == cudaSuccess && g_last_error[0] == 0) ? MIE_OK : MIE_ERR_CUDA;
}

const char* mie_last_cuda_error(void) { return g_last_error; }

int mie_moe_route(const mie_moe_args* a, void* stream) {
  if (!a) return MIE_ERR_INVALID;
  return run_moe(*a, static_cast<cudaStream_t>(stream), false, true);
}

int mie_moe_decode(const mie_moe_args* a, void* stream) {
  if (!a) return MIE_ERR_INVALID;
  return run_moe(*a, static_cast<cudaStream_t>(stream), false, false);
}

int mie_attn_decode(const mie_attn_args* a, void* stream) {
  if (!a) return MIE_ERR_INVALID;
  return run_attn(*a, static_cast<cudaStream_t>(stream), false);
}

int mie_attn_decode_fixed_scratch(const mie_attn_args* a, void* stream) {
  if (!a) return MIE_ERR_INVALID;
  // the partials of a deferred merge would stay in the library's array, where
  // no consumer can read them: refused
  if (a->defer_merge) return MIE_ERR_INVALID;
  // the request itself first, then the size limit, then the one-time set-up
  int rc = check_attn(*a, false);
  if (rc) return rc;
  mie_attn_args v = *a;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  rc = attn_fixed_scratch_bind(&v, st);  // partials + counters from the fixed array
  if (rc) return rc;
  return run_attn(v, st, false);
}

int mie_qkv_rope_store(const mie_qkv_args* a, void* stream) {
  if (!a) return MIE_ERR_INVALID;
  return run_qkv(*a, static_cast<cudaStream_t>(stream), false);
}

int mie_proj_residual(const mie_proj_args* a, void* stream) {
  if (!a) return MIE_ERR_INVALID;
  return run_proj(*a, static_cast<cudaStream_t>(stream), false);
}

int mie_lmhead_argmax(const mie_lmhead_args* a, void* stream) {
  if (!a) return MIE_ERR_INVALID;
  return run_lmhead(*a, static_cast<cudaStream_t>(stream), false);
}

int mie_gemm(const mie_gemm_args* a, void* stream) {
  if (!a) return MIE_ERR_INVALID;
  return gemm_run(*a, static_cast<cudaStream_t>(stream));
}

int mie_prefill_norm(const mie_prefill_norm_args* a, void* stream) {
  return a ? prefill_norm(*a, static_cast<cudaStream_t>(stream)) : MIE_ERR_INVALID;
}
int mie_prefill_rope_kv(const mie_prefill_rope_args* a, void* stream) {
  return a ? prefill_rope_kv(*a, static_cast<cudaStream_t>(stream)) : MIE_ERR_INVALID;
}
int mie_prefill_route(const mie_prefill_route_args* a, void* stream) {
  return a ? prefill_route(*a, static_cast<cudaStream_t>(stream)) : MIE_ERR_INVALID;
}
int mie_prefill_combine(const mie_prefill_combine_args* a, void* stream) {
  return a ? prefill_combine(*a, static_cast<cudaStream_t>(stream)) : MIE_ERR_INVALID;
}
int mie_prefill_attention(const mie_prefill_attn_args* a, void* stream) {
  return a ? prefill_attention(*a, static_cast<cudaStream_t>(stream)) : MIE_ERR_INVALID;
}

// ---- expert-parallel all-reduce over peer memory ----
int64_t mie_peer_buffer_bytes(int n, int world) {
  return (n < 1 || world < 1 || world > MIE_PEER_MAX_RANKS) ? 0 : peer_buffer_bytes(n, world);
}

int mie_peer_reduce(const mie_peer_reduce_args* a, void* stream) {
  return a ? peer_reduce(*a, static_cast<cudaStream_t>(stream)) : MIE_ERR_INVALID;
}

int mie_peer_alloc(int64_t bytes, void** ptr) {
  if (!ptr || bytes <= 0) return MIE_ERR_INVALID;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, (size_t)bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();  // zeroed before any stream uses it (one-time set-up)
  if (e != cudaSuccess) {
    note_cuda_error(e, "mie_peer_alloc");
    if (p) cudaFree(p);
    return MIE_ERR_CUDA;
  }
  *ptr = p;
  return MIE_OK;
}

int mie_peer_free(void* ptr) {
  if (!ptr) return MIE_ERR_INVALID;
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) note_cuda_error(e, "mie_peer_free");
  return e == cudaSuccess ? MIE_OK : MIE_ERR_CUDA;
}

int mie_peer_handle(const void* ptr, void* handle64) {
  if (!ptr || !handle64) return MIE_ERR_INVALID;
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "64-byte IPC handle");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e != cudaSuccess) {
    note_cuda_error(e, "mie_peer_handle");
    return MIE_ERR_CUDA;
  }
  memcpy(handle64, &h, sizeof(h));
  return MIE_OK;
}

int mie_peer_open(const void* handle64, void** ptr) {
  if (!handle64 || !ptr) return MIE_ERR_INVALID;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    note_cuda_error(e, "mie_peer_open");
    return MIE_ERR_CUDA;
  }
  *ptr = p;
  return MIE_OK;
}

int mie_peer_close(void* ptr) {
  if (!ptr) return MIE_ERR_INVALID;
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) note_cuda_error(e, "mie_peer_close");
  return e == cudaSuccess ? MIE_OK : MIE_ERR_CUDA;
}

int mie_decode_layer(const mie_step_desc* d, int l, void* stream) {
  if (!d || l < 0 || l >= d->num_layers) return MIE_ERR_INVALID;
  int rc = check_step(*d);
  if (rc) return rc;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool pdl = d->use_pdl != 0;
  if ((rc = run_qkv(step_qkv(*d, l), st, pdl))) return rc;
  if ((rc = run_attn(step_attn(*d, l), st, pdl))) return rc;
  if ((rc = run_proj(step_proj(*d, l), st, pdl))) return rc;
  return run_moe(step_moe(*d, l), st, pdl, false);
}

int mie_decode_head(const mie_step_desc* d, void* stream) {
  if (!d) return MIE_ERR_INVALID;
  if (d->sample_temperature > 0.f) return MIE_ERR_UNSUPPORTED;  // the device sampler is in the persistent step
  const int rc = check_step(*d);
  if (rc) return rc;
  return run_lmhead(step_lmhead(*d), static_cast<cudaStream_t>(stream), d->use_pdl != 0);
}

int mie_decode_step(const mie_step_desc* d, void* stream) {
  if (!d) return MIE_ERR_INVALID;
  if (d->step_scratch) {
    StepPlan plan;
    const int rc = persistent_geometry(*d, &plan);
    if (rc) return rc;
    if (d->step_scratch_bytes < plan.words() * (int64_t)sizeof(uint64_t)) return MIE_ERR_INVALID;
    if (plan.cluster) return cstep_launch(*d, plan.cg, d->step_scratch, static_cast<cudaStream_t>(stream));
    return step_launch(*d, plan.g, d->step_scratch, static_cast<cudaStream_t>(stream));
  }
  if (d->sample_temperature > 0.f) return MIE_ERR_UNSUPPORTED;  // before any launch
  if (d->start_gate) return MIE_ERR_UNSUPPORTED;  // the start gate is a persistent-step feature
  for (int l = 0; l < d->num_layers; ++l) {
    const int rc = mie_decode_layer(d, l, stream);
    if (rc) return rc;
  }
  return mie_decode_head(d, stream);
}

int mie_step_kernel_of(const mie_step_desc* d) {
  if (!d) return -MIE_ERR_INVALID;
  StepPlan plan;
  const int rc = persistent_geometry(*d, &plan);
  if (rc) return -rc;
  return plan.cluster ? MIE_STEP_CLUSTER : MIE_STEP_FLAT;
}

int64_t mie_step_scratch_bytes(const mie_step_desc* d) {
  if (!d) return -MIE_ERR_INVALID;
  StepPlan plan;
  const int rc = persistent_geometry(*d, &plan);
  if (rc) return -(int64_t)rc;
  return plan.words() * (int64_t)sizeof(uint64_t);
}

}  // extern "C"
