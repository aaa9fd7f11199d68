// Internal host-side interface between the kernel files and the C ABI layer.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <utility>

#include "../../include/mie.h"

namespace mie {

// Record a failed CUDA call (readable through mie_last_cuda_error()).
void note_cuda_error(cudaError_t e, const char* what);

// Shared-memory layout of the MoE kernel (byte offsets into dynamic smem).
struct MoeLayout {
  uint32_t off_h, off_res;  // offsets in floats: expert activations [2, Hx], down results [2, max_rows]
  uint32_t smem;            // dynamic shared memory bytes
  int max_rows;             // down-phase rows per CTA (upper bound)
  int route_only;           // 1: stop after routing (mie_moe_route)
};

// Shared-memory layout of the single-vector GEMV kernels (QKV, proj, LM head):
// only the fp32 input vector lives in dynamic shared memory.
struct GemvLayout {
  uint32_t smem;
};

struct AttnLayout {
  uint32_t off_bar, off_kv, off_q, off_p, off_acc, smem;
  int nstage;
  int stage_tokens;  // tokens per stage (a multiple of block_size)
  // the cp.async kernel (16-byte K/V rows): tokens per chunk buffer, block
  // ids of one split cached in shared memory, their offset
  int fast, chunk_tok, cap_blocks;
  uint32_t off_blk;
};

// Dynamic shared memory any layout here may use (under the 227 KB opt-in
// limit minus the kernels' static shared memory).
constexpr int kMaxDynSmem = 220 * 1024;

// ---- persistent decode step (step.cu) ----
constexpr int kStepThreads = 512;                   // one CTA of 16 warps per SM
constexpr int kMaxStepLayers = 48;                  // layer descriptors carried in the launch parameters
constexpr uint32_t kStepKvChunkBytes = 32 * 1024;   // K+V of one split staged in shared memory at a time
constexpr int kStepHeadStagesMax = 8;               // LM-head ring stages
constexpr uint32_t kStepMaxSmem = 223 * 1024;       // dynamic shared memory of the step kernel (static: < 4 KB)
constexpr int kStepTopKMax = 64;                    // largest top_k of the device sampler
constexpr int kStepMaxExpertHidden = 4096;          // expert hidden size of the persistent step
constexpr int kStepHeadRowsMax = 512;               // LM-head rows of one CTA the top-k sampler sorts

// Geometry of one persistent step launch: exchange-buffer offsets (64-bit
// words into the caller's scratch) and the shared-memory layout (bytes).
struct StepGeom {
  uint64_t* ll;   // scratch base
  int64_t words;  // scratch size in 64-bit words
  int64_t off_a[2], off_b[2], off_c[2], off_d[2], off_e[2];
  int64_t off_cand;  // sampling with top-k: kStepTopKMax candidates per CTA
  int G;          // CTAs (one per SM)
  int S;          // attention splits per head
  int natt;       // attention CTAs (num_heads * S)
  int chunk_tok;  // K/V tokens per shared-memory chunk
  int q_stage;    // q rows of the head staged in shared memory (the rest are read from global memory)
  int moe_staged; // 1: the selected experts' rows are staged in shared memory
  int wide;       // 1: the wide kernel variant (any head_dim piece count, long expert rows)
  int head_bias_smem;  // 1: the CTA's LM-head bias values fit in the h vector's shared memory
  int nr_max;     // out_proj / down rows of one CTA (upper bound)
  int head_rows, head_stages;  // LM-head ring: rows per stage, stages
  int head_early;               // ring stages inside the attention staging area
  // shared memory (byte offsets): fp32 vectors (x, normalised x, x_mid, expert
  // activations, attention output, q + this CTA's k / v values, scratch,
  // scores), the attention norm weights, the attention staging area sm_qw ..
  // sm_kv + K/V chunk (reused as the LM-head ring), and sm_moe (out_proj rows,
  // router, MoE norm weights; after routing the selected experts' rows)
  uint32_t sm_x, sm_xn, sm_xm, sm_h, sm_o, sm_qk, sm_acc, sm_sc, sm_anw;
  uint32_t sm_qw, sm_kvw, sm_kv, sm_moe, smem;
};

struct StepParams {
  mie_step_desc d;  // d.layers is not used on the device
  StepGeom g;
  mie_layer_desc layers[kMaxStepLayers];
};

// ---- persistent decode step on thread-block clusters (step_cluster.cu) ----
constexpr int kStepCluster = 6;   // CTAs per cluster = attention splits per head
constexpr int kClusterHeadDim = 64;  // head_dim of the cluster step

// Geometry of one cluster-step launch: exchange-buffer offsets (64-bit words
// into the caller's scratch) and the shared-memory layout (bytes).
struct CGeom {
  uint64_t* ll;   // scratch base
  int64_t words;  // scratch size in 64-bit words
  int64_t off_x[2], off_p[2], off_h[2];  // x of a layer [D], out_proj partials [H, D], expert hidden [2 Hx]
  int G, NC;      // CTAs, clusters (G = NC * kStepCluster)
  int chunk_tok;  // K/V tokens per shared-memory chunk
  int np_max, nv_max;  // RoPE pairs / v rows of one split (upper bounds)
  int orows;      // out_proj rows of one split (upper bound; the tile height)
  int nu_max, nr_max;  // up units / down rows of one CTA (upper bounds)
  int head_rows, head_stages;  // LM-head ring
  // staging regions: A (q/k/v rows, then the selected experts' gate/up rows),
  // K (K then V chunk), O (out_proj tile), D (down rows), R (router + norms);
  // [sm_k, sm_fn) is the LM-head ring after the last layer
  uint32_t sm_a, sm_k, sm_o, sm_d, sm_r;
  // fp32 vectors: x, normalised x, x_mid [2][D], x_mid square sums [2][CS],
  // gathered q / k_new / v_new [2][3][hd], merge partials [2][CS][hd + 4],
  // own q/k/v GEMV results, scores, scratch, expert hidden [2 Hx], received
  // partials [H + 1][orows], merged o [hd], router partials [2][CS][E]
  uint32_t sm_x, sm_xn, sm_xm, sm_ss, sm_g, sm_mg, sm_qkv, sm_sc, sm_ab, sm_h, sm_pr, sm_ov, sm_rp;
  uint32_t sm_fn;  // final norm weights
  uint32_t smem;
  // expert parallel (peer_world > 1): this rank, every rank's exchange buffer
  // as this process maps it ([2 layer parities][world][D] tagged words) and
  // the group's device step counter, whose value + 1 keys the step's tags
  int peer_rank, peer_world;
  uint64_t* peer_bufs[MIE_PEER_MAX_RANKS];
  uint32_t* peer_seq;
  // int8 experts (qbits 8; 0: bf16): log2 of the group size, and where the
  // staged rows' fp32 group scales start in regions A and D (bytes)
  int qbits, qgsh;
  uint32_t q_a_scale, q_d_scale;
};

struct CStepParams {
  mie_step_desc d;  // d.layers is not used on the device
  CGeom g;
  mie_layer_desc layers[kMaxStepLayers];
  CUtensorMap omap[kMaxStepLayers];  // per layer: out_proj [D, D] bf16, box hd x orows
};

// Allow the largest dynamic shared memory the device permits next to the
// kernel's static shared memory.
template <typename Kernel>
inline void set_max_smem(Kernel k) {
  int dev = 0, optin = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  cudaFuncAttributes fa{};
  cudaError_t e = cudaFuncGetAttributes(&fa, reinterpret_cast<const void*>(k));
  if (e != cudaSuccess) {
    note_cuda_error(e, "cudaFuncGetAttributes");
    return;
  }
  e = cudaFuncSetAttribute(reinterpret_cast<const void*>(k), cudaFuncAttributeMaxDynamicSharedMemorySize,
                           optin - (int)fa.sharedSizeBytes);
  if (e != cudaSuccess) note_cuda_error(e, "cudaFuncSetAttribute(MaxDynamicSharedMemorySize)");
}

// Launch with optional programmatic dependent launch.  Returns MIE_OK or MIE_ERR_CUDA.
template <typename... KArgs, typename... Args>
inline int launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, uint32_t smem, cudaStream_t stream, bool pdl,
                  Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess) {
    note_cuda_error(e, "cudaLaunchKernelEx");
    return MIE_ERR_CUDA;
  }
  return MIE_OK;
}

// moe.cu
MoeLayout moe_layout(const mie_moe_args& a, int grid, int slot_bytes, int nslot);
int moe_decode_launch(const mie_moe_args& a, const MoeLayout& L, int grid, cudaStream_t st, bool pdl);
void moe_set_attributes();
int moe_decode_q_launch(const mie_moe_args& a, const MoeLayout& L, int grid, cudaStream_t st, bool pdl);
void moe_q_set_attributes();
int64_t peer_buffer_bytes(int n, int world);
int peer_reduce(const mie_peer_reduce_args& a, cudaStream_t st);

// attention.cu
AttnLayout attn_layout(const mie_attn_args& a);
int attn_decode_launch(const mie_attn_args& a, const AttnLayout& L, cudaStream_t st, bool pdl);
void attn_set_attributes();
int attn_fixed_scratch_bind(mie_attn_args* a, cudaStream_t st);

// gemv.cu
GemvLayout qkv_layout(const mie_qkv_args& a, int grid);
int qkv_launch(const mie_qkv_args& a, const GemvLayout& L, int grid, cudaStream_t st, bool pdl);
GemvLayout proj_layout(const mie_proj_args& a, int grid);
int proj_launch(const mie_proj_args& a, const GemvLayout& L, int grid, cudaStream_t st, bool pdl);
GemvLayout lmhead_layout(const mie_lmhead_args& a, int grid);
int lmhead_launch(const mie_lmhead_args& a, const GemvLayout& L, int grid, cudaStream_t st, bool pdl);
void gemv_set_attributes();

// step.cu
int step_geometry(const mie_step_desc& d, int grid, StepGeom* g);
int step_launch(const mie_step_desc& d, const StepGeom& g, uint64_t* scratch, cudaStream_t st);
void step_set_attributes();
// step_cluster.cu: MIE_OK when the cluster step takes `d` (and fills *g)
int cstep_geometry(const mie_step_desc& d, CGeom* g);
int cstep_launch(const mie_step_desc& d, const CGeom& g, uint64_t* scratch, cudaStream_t st);
void cstep_set_attributes();
// gemm.cu: cuTensorMapEncodeTiled through the runtime's driver entry point
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn();
// step_wide.cu (the wide variant of the persistent step, its own translation unit)
int step_launch_wide(const StepParams& p, cudaStream_t st);
void step_set_attributes_wide();

// gemm.cu (prefill GEMM on the tensor cores)
enum {
  kEpiF32 = MIE_GEMM_F32,
  kEpiBF16 = MIE_GEMM_BF16,
  kEpiResid = MIE_GEMM_RESID,
  kEpiSwiGLU = MIE_GEMM_SWIGLU,
  kEpiGelu = MIE_GEMM_GELU
};
// Device-side arguments of one GEMM launch (the tensor maps travel separately).
struct GemmArgs {
  int M, N, K;
  void* c;
  int64_t ldc;
  const float* resid;
  int64_t ldr;
  const int32_t* counts;
  int a_group_rows, b_group_rows, c_group_rows;
  int32_t* status;
  const __nv_bfloat16* bias;
  int64_t bias_group_stride;
};
int gemm_run(const mie_gemm_args& a, cudaStream_t st);
void gemm_set_attributes();
// prefill.cu
int prefill_norm(const mie_prefill_norm_args& a, cudaStream_t st);
int prefill_rope_kv(const mie_prefill_rope_args& a, cudaStream_t st);
int prefill_route(const mie_prefill_route_args& a, cudaStream_t st);
int prefill_combine(const mie_prefill_combine_args& a, cudaStream_t st);
int prefill_attention(const mie_prefill_attn_args& a, cudaStream_t st);

int num_sms();

}  // namespace mie
