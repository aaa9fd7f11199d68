/*
 * mie.h -- C ABI of the B200 (sm_100a) batch-one decode kernels for the
 * miniMoE engine.  Plain C: device pointers, sizes and a cudaStream_t passed
 * as void*.  No torch types cross this boundary.
 *
 * Every entry point returns an int status (MIE_OK == 0).  Kernels also record
 * device-side failures (bounded waits that gave up, out-of-range block ids,
 * positions or expert ids) in an optional device status word, which the host
 * reads after synchronising; no kernel traps.
 *
 * Reference interfaces replaced (paths relative to the reference project):
 *   mie_moe_route        <- src/moe_engine/fused_moe.py:274-309  (route)
 *   mie_moe_decode       <- src/moe_engine/fused_moe.py:312-380  (decode)
 *   mie_attn_decode      <- src/moe_engine/paged_attention.py:113-154 (decode),
 *                           and the contiguous SDPA decode at model.py:261-266
 *   mie_qkv_rope_store   <- src/moe_engine/model.py:226-234,247 (QKV projection,
 *                           head split, cache write) plus the norm at
 *                           model.py:495 and embedding at model.py:557-558
 *   mie_proj_residual    <- src/moe_engine/model.py:268-269,495 (out_proj + residual)
 *   mie_lmhead_argmax    <- src/moe_engine/model.py:564-565,600-603 (final norm,
 *                           tied LM head, greedy argmax)
 *   mie_decode_step      <- src/moe_engine/model.py:543-565 (Model.forward for one
 *                           decode token) as one launch sequence, or as one
 *                           persistent launch (mie_step_scratch_bytes)
 *   mie_gemm             <- the prompt prefill's projections: F.linear of the
 *                           QKV and out projections (model.py:226-234,268) and
 *                           the expert matmuls of the reference MoE loop
 *                           (model.py:443-461), on the tcgen05 tensor cores
 *   mie_prefill_norm     <- model.py:491-492,557-558 (embedding + norms, T tokens)
 *   mie_prefill_rope_kv  <- model.py:226-247 (head split, RoPE, cache write)
 *   mie_prefill_route    <- model.py:443-452 (fp32 router, top-2, softmax) plus
 *                           the per-expert token selection of the loop
 *   mie_prefill_combine  <- model.py:453-461 (weighted index_add_ of expert outputs)
 *   mie_prefill_attention <- model.py:252-256 (causal SDPA of the prefill fast path)
 * No counterpart in the reference (it is a single-GPU engine without quantized
 * weights): mie_peer_reduce (the expert-parallel all-reduce over peer memory),
 * the quantized-expert fields of mie_moe_args (its roadmap item,
 * moe-inference-engine.md:36), mie_attn_decode_fixed_scratch.
 */
#ifndef MIE_H
#define MIE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
enum {
  MIE_OK = 0,
  MIE_ERR_INVALID = 1,      /* bad argument (null pointer, bad size, misalignment) */
  MIE_ERR_UNSUPPORTED = 2,  /* shape / dtype combination has no kernel */
  MIE_ERR_CUDA = 3,         /* a CUDA runtime call failed */
  MIE_ERR_TIMEOUT = 4,      /* device: a bounded wait gave up */
  MIE_ERR_RANGE = 5,        /* device: block id / position / expert / token out of range */
  MIE_ERR_SCRATCH_LIMIT = 6 /* request larger than the fixed scratch of mie_attn_decode_fixed_scratch */
};

/* element types */
enum { MIE_F32 = 0, MIE_BF16 = 1 };
/* ranks of an expert-parallel group served by the all-reduce over peer memory */
#define MIE_PEER_MAX_RANKS 8
/* normalisation applied in a kernel prologue */
enum { MIE_NORM_NONE = 0, MIE_NORM_RMS = 1, MIE_NORM_LAYER = 2 };
/* expert activation */
enum { MIE_ACT_GELU = 0, MIE_ACT_SWIGLU = 1 };

/* Fused top-2 MoE decode: norm -> router GEMV -> top-2 (ties to the lower id)
 * -> 2-way softmax -> selected experts' up GEMVs + activation -> down GEMVs ->
 * weighted combine (+ residual).  One persistent launch. */
typedef struct mie_moe_args {
  int dtype;              /* weights */
  int x_dtype;            /* x */
  int out_dtype;          /* out */
  int hidden_dim;         /* D */
  int expert_hidden_dim;  /* Hx */
  int num_experts;        /* E <= 32 */
  int top_k;              /* must be 2 */
  int act;                /* MIE_ACT_* */
  int norm;               /* MIE_NORM_* applied to x before routing */
  float eps;
  const void* x;          /* [D] */
  const void* norm_w;     /* [D] or NULL */
  const void* norm_b;     /* [D] or NULL */
  const void* router_w;   /* [E, D] */
  const void* w1;         /* [E', Hx, D]: GELU fc1 / SwiGLU gate */
  const void* b1;         /* [E', Hx] or NULL */
  const void* w3;         /* [E', Hx, D]: SwiGLU up, NULL for GELU */
  const void* w2;         /* [E', D, Hx]: down */
  const void* b2;         /* [E', D] or NULL */
  float* router_logits;   /* [E] fp32 out, or NULL */
  int32_t* expert_ids;    /* [2] out, or NULL */
  float* route_weights;   /* [2] fp32 out, or NULL */
  float* hidden;          /* scratch [2, Hx] fp32 */
  void* out;              /* [D]: out = (residual ? x : 0) + moe */
  int residual;
  uint32_t* sync;         /* 4 words, zeroed once by the caller, reused forever */
  int32_t* status;        /* device status word, or NULL */
  const int32_t* skip;    /* device flag: nonzero -> do nothing; or NULL */
  int grid;               /* CTAs; 0 = one per SM */
  int expert_base;        /* expert parallel: weights hold experts [base, base+count) */
  int expert_count;       /* 0 = all experts local */
  /* Quantized experts (no counterpart in the reference; its roadmap item
   * moe-inference-engine.md:36).  0: w1 / w3 / w2 hold `dtype` values.  8 or 4:
   * they hold int8 values, or int4 values two per byte (the even element in
   * the low nibble), of rows quantized in groups of group_size consecutive
   * elements along the row (symmetric: w = scale * q, |q| <= 127 or 7); the
   * router, biases and activations stay in `dtype`.  Rows must be multiples
   * of 16 bytes and of group_size (a power of two, at least 32). */
  int expert_bits;
  int group_size;
  const float* w1_scale;  /* [E', Hx, D / group_size] */
  const float* w3_scale;  /* [E', Hx, D / group_size] (SwiGLU) */
  const float* w2_scale;  /* [E', D, Hx / group_size] */
  /* Expert parallel with the all-reduce fused in (peer_world > 1; no
   * counterpart in the reference): each CTA stores its output rows' partial
   * -- its local experts' weighted sum -- as tagged words into every rank's
   * receive buffer (the layout, call counter and call-order rules of
   * mie_peer_reduce, n = hidden_dim), polls its own buffer for the same rows
   * and writes out = (residual ? x : 0) + the rank-order sum. */
  int peer_rank;
  int peer_world;                          /* 0 or 1: no exchange */
  uint32_t* peer_seq;
  uint64_t* peer_bufs[MIE_PEER_MAX_RANKS];
  int64_t peer_wait_limit_ns;              /* 0: 200 ms */
} mie_moe_args;

/* Single-query attention over a paged ([nb, H, bs, hd] per layer) or
 * contiguous ([H, S, hd] per layer) K/V cache, split-K over KV blocks with a
 * log-sum-exp merge in the same launch (last CTA per head merges). */
typedef struct mie_attn_args {
  int kv_dtype;
  int q_dtype;
  int out_dtype;
  int num_heads;
  int head_dim;           /* 4..128, multiple of 4 */
  const void* q;          /* [H, hd] */
  const void* k;          /* layer base */
  const void* v;          /* layer base */
  const int32_t* block_table; /* paged: [>= ceil(ctx/bs)] physical ids; NULL: contiguous */
  int num_blocks;         /* paged: blocks in the pool (range check) */
  int block_size;         /* paged: tokens per block; contiguous: tile tokens */
  int64_t stride_block;   /* elements between blocks (contiguous: block_size*stride_tok) */
  int64_t stride_head;    /* elements between heads */
  int64_t stride_tok;     /* elements between tokens (== head_dim) */
  int ctx_len;            /* context length when ctx_dev is NULL */
  const int32_t* ctx_dev; /* device position p: ctx = *ctx_dev + ctx_dev_offset */
  int ctx_dev_offset;
  int max_ctx;            /* upper bound for ctx (range check) */
  float scale;            /* softmax scale, normally 1/sqrt(hd) */
  void* out;              /* [H, hd] */
  float* partials;        /* scratch [H, max_splits, hd + 2] fp32 */
  uint32_t* counters;     /* [H], zeroed once by the caller */
  int splits;             /* KV splits per head (>= 1) */
  int max_splits;
  int new_token_last;     /* 1: the last token was written by the preceding kernel */
  int32_t* status;
  const int32_t* skip;
  int defer_merge;        /* 1: write every split's (m, l, acc) to partials and leave the
                             merge to the consumer (mie_proj_args.attn_partials) */
} mie_attn_args;

/* Norm + QKV GEMV + RoPE + K/V store into the cache slot of the device
 * position.  Optionally gathers the token embedding first (layer 0). */
typedef struct mie_qkv_args {
  int dtype;              /* weights / embeddings */
  int kv_dtype;
  int hidden_dim;
  int num_heads;
  int head_dim;
  int norm;
  float eps;
  const void* norm_w;
  const void* norm_b;
  float* x;               /* fp32 residual stream [D] */
  const float* x_add;     /* pending residual delta [D] or NULL (x := x + x_add) */
  const void* embedding;  /* [V, D] or NULL; when set x := emb[*token] (+ pos_emb[pos]) */
  const void* pos_embedding; /* [S, D] or NULL */
  const int64_t* token;
  int vocab;
  const void* w;          /* [3D, D] */
  const void* b;          /* [3D] or NULL */
  const float* rope_cos;  /* [S, hd/2] or NULL (no RoPE) */
  const float* rope_sin;
  const int32_t* pos;     /* device position of the new token */
  int max_pos;
  float* q_out;           /* [H*hd] fp32 */
  void* k_cache;          /* layer base */
  void* v_cache;
  const int32_t* block_table; /* NULL: contiguous */
  int num_blocks;
  int block_size;
  int64_t stride_block;
  int64_t stride_head;
  int64_t stride_tok;
  int32_t* status;
  const int32_t* skip;
  int grid;
} mie_qkv_args;

/* out[r] = (accumulate ? out[r] : 0) + add[r] + W[r,:] . in + b[r]  (fp32 in/out). */
typedef struct mie_proj_args {
  int dtype;
  int rows;
  int cols;
  const void* w;
  const void* b;
  const float* in;
  float* out;
  const float* add;       /* [rows] or NULL */
  int accumulate;
  int32_t* status;
  const int32_t* skip;
  int grid;
  /* Optional: build `in` by merging split-K attention partials ([heads, max_splits,
   * head_dim + 2] as written with mie_attn_args.defer_merge) instead of reading it. */
  const float* attn_partials;
  int attn_heads;
  int attn_head_dim;
  int attn_splits;
  int attn_max_splits;
} mie_proj_args;

/* Final norm + tied LM-head GEMV + argmax (ties to the lower id), with the
 * step's device-side bookkeeping (next token, position, EOS flag, token log). */
typedef struct mie_lmhead_args {
  int dtype;
  int vocab;
  int hidden_dim;
  int norm;
  float eps;
  const void* norm_w;
  const void* norm_b;
  const float* x;
  const float* x_add;
  const void* w;          /* [V, D] */
  const void* b;          /* [V] or NULL */
  float* logits;          /* [V] fp32 or NULL */
  float* partial_val;     /* scratch [grid] */
  int32_t* partial_idx;   /* scratch [grid] */
  uint32_t* counter;      /* 1 word, zeroed once */
  int64_t* token_out;     /* argmax id */
  int32_t* pos;           /* incremented by one when non-NULL */
  int64_t* tokens_log;    /* optional append log [log_capacity] */
  int32_t* log_count;
  int log_capacity;
  int32_t* done;          /* set to 1 when the token equals eos_id (if non-NULL) */
  int eos_id;
  int32_t* status;
  const int32_t* skip;
  int grid;
} mie_lmhead_args;

/* Per-layer weights and cache bases for mie_decode_step. */
typedef struct mie_layer_desc {
  const void* attn_norm_w;
  const void* attn_norm_b;
  const void* qkv_w;
  const void* qkv_b;
  const void* out_w;
  const void* out_b;
  const void* moe_norm_w;
  const void* moe_norm_b;
  const void* router_w;
  const void* w1;
  const void* b1;
  const void* w3;
  const void* w2;
  const void* b2;
  void* k_cache;
  void* v_cache;
  /* quantized experts (mie_step_desc.expert_bits set): w1 / w3 / w2 hold the
   * int8 values or packed int4 pairs, these their fp32 group scales
   * ([experts, rows, cols / group_size], as mie_moe_args) */
  const float* w1_scale;
  const float* w3_scale;
  const float* w2_scale;
} mie_layer_desc;

/* One whole decode step (all layers + LM head) for one token. */
typedef struct mie_step_desc {
  int dtype;
  int kv_dtype;
  int num_layers;
  int hidden_dim;
  int num_heads;
  int head_dim;
  int num_experts;
  int top_k;
  int expert_hidden_dim;
  int vocab;
  int norm;
  int act;
  float eps;
  float attn_scale;
  int max_pos;
  const mie_layer_desc* layers;  /* host array [num_layers] */
  const void* embedding;
  const void* pos_embedding;
  const void* final_norm_w;
  const void* final_norm_b;
  const void* lm_bias;
  const float* rope_cos;
  const float* rope_sin;
  const int32_t* block_table;    /* NULL: contiguous cache */
  int num_blocks;
  int block_size;
  int64_t kv_stride_block;
  int64_t kv_stride_head;
  int64_t kv_stride_tok;
  int64_t* token;                /* device: input token, overwritten by the argmax */
  int32_t* pos;                  /* device: position of the input token */
  int32_t* done;                 /* device EOS flag or NULL */
  int eos_id;
  int64_t* tokens_log;
  int32_t* log_count;
  int log_capacity;
  float* x;                      /* scratch fp32 [D] */
  float* q;                      /* scratch fp32 [H*hd] */
  float* attn_out;               /* scratch fp32 [H*hd] */
  float* moe_hidden;             /* scratch fp32 [2, Hx] */
  float* moe_partial;            /* expert parallel: MoE contribution [D] or NULL */
  int expert_base;
  int expert_count;
  float* attn_partials;          /* scratch [H, max_splits, hd+2] */
  uint32_t* attn_counters;       /* [H] zeroed once */
  uint32_t* moe_sync;            /* [4] zeroed once */
  float* lm_partial_val;         /* [lm_grid] */
  int32_t* lm_partial_idx;       /* [lm_grid] */
  uint32_t* lm_counter;          /* [1] zeroed once */
  float* logits;                 /* [V] or NULL */
  int32_t* status;
  int attn_splits;
  int max_splits;
  int lm_grid;                   /* 0 = one per SM */
  int use_pdl;                   /* programmatic dependent launch between kernels */
  /* Persistent step: when non-NULL, mie_decode_step runs the whole step as ONE
   * launch of one CTA per SM whose phases exchange their results through this
   * buffer (see mie_step_scratch_bytes).  Zeroed by the caller once, reused
   * for every step; zero it again after a step reported a device failure. */
  uint64_t* step_scratch;
  int64_t step_scratch_bytes;
  /* Sampling instead of greedy argmax (model.py:604-613), persistent step only
   * (the per-op launch sequence returns MIE_ERR_UNSUPPORTED for it): with
   * sample_temperature > 0 the token is drawn from softmax(logits / T),
   * restricted to the logits >= the sample_top_k-th largest when
   * 0 < sample_top_k <= 64 (all logits when sample_top_k <= 0), by the
   * Gumbel-max rule with a counter-based random stream keyed by
   * (*sample_seed, position, token id). */
  float sample_temperature;
  int sample_top_k;
  const uint64_t* sample_seed;  /* device word, read every step */
  /* Persistent step: when non-NULL (with log_count), a step whose *log_count
   * has reached *step_limit changes nothing, like a step after EOS -- so a
   * graph of several step launches decodes at most *step_limit tokens.  With
   * use_pdl the launch is programmatic-dependent: the next step's CTAs stage
   * their first weights while this step's last CTA finishes the LM head. */
  const int32_t* step_limit;
  /* Persistent step: every wait on another CTA's result or on a bulk copy
   * gives up after this many nanoseconds (0: the default, 200 ms); the step
   * then ends with MIE_ERR_TIMEOUT in *status and the caller zeroes
   * step_scratch before the next step. */
  int64_t wait_limit_ns;
  /* Persistent step: when non-NULL, the step starts only once *start_gate is
   * nonzero -- a flag written by another stream, a peer GPU or the host
   * through mapped memory, for a step queued ahead of the input it reads.  A
   * gate still closed after wait_limit_ns ends the step with MIE_ERR_TIMEOUT
   * before it changes anything. */
  const int32_t* start_gate;
  /* Which persistent step kernel runs the step (step_scratch set):
   * MIE_STEP_AUTO picks the cluster kernel when it takes the shapes, else the
   * one-CTA-per-SM kernel; the other two force one (MIE_ERR_UNSUPPORTED when
   * the forced kernel cannot take the shapes). */
  int step_kernel;
  /* Expert parallel over the ranks of mie_peer_reduce_args (a host pointer,
   * read at launch; n = hidden_dim; in, out and status unused):
   * - per-layer launch sequence (moe_partial set): each layer's MoE kernel
   *   completes the all-reduce of its partial itself over these peer
   *   buffers (see the peer_* fields of mie_moe_args), so moe_partial
   *   receives the sum over ranks;
   * - persistent step (step_scratch set, moe_partial NULL, world > 1; the
   *   cluster kernel only): the layers' weights hold experts
   *   [expert_base, expert_base + expert_count); the step computes the
   *   selected experts among them and completes every layer's all-reduce
   *   inside the kernel -- the rank's partial of each output row is stored
   *   into every rank's buffer, every reader sums the ranks' words in rank
   *   order onto x_mid.  Every rank runs the same steps on the same token;
   *   *seq advances once per step.  A wait for a peer's words gives up after
   *   wait_limit_ns (MIE_ERR_TIMEOUT); the ranks' exchange state then
   *   differs, so the group makes new buffers and a new counter. */
  const struct mie_peer_reduce_args* moe_peer;
  /* Quantized experts (0: the layers' experts are in `dtype`): 8 or 4 with
   * group_size as in mie_moe_args, scales in the layer descriptors.  The
   * cluster step takes int8 (bf16 model, group_size a power of two >= 32
   * dividing hidden_dim and expert_hidden_dim); int4, and int8 on other
   * shapes, run the per-layer launch sequence. */
  int expert_bits;
  int group_size;
} mie_step_desc;

enum { MIE_STEP_AUTO = 0, MIE_STEP_FLAT = 1, MIE_STEP_CLUSTER = 2 };

/* Prefill GEMM on the tcgen05 tensor cores: C = A . B^T with A [M, K] and
 * B [N, K] bf16 row-major (rows of K elements), fp32 accumulation, then one of
 * the epilogues below.  K a multiple of 64, N a multiple of 128, rows 16-byte
 * aligned.  Grouped form (groups > 1 or counts set): group g uses A rows
 * [g a_group_rows, ..), B rows [g b_group_rows, ..) and C rows
 * [g c_group_rows, ..); only its first counts[g] rows (a device array; M when
 * counts is NULL, at most M) are computed and stored. */
enum {
  MIE_GEMM_F32 = 0,    /* C fp32 */
  MIE_GEMM_BF16 = 1,   /* C bf16 */
  MIE_GEMM_RESID = 2,  /* C fp32 = resid + A.B^T (resid may alias C) */
  MIE_GEMM_SWIGLU = 3, /* B = gate rows, b2 = up rows; N counts gate + up
                          columns; C bf16 [.., N / 2] = silu(A.B^T) * (A.B2^T) */
  MIE_GEMM_GELU = 4    /* C bf16 = gelu_erf(A.B^T + bias) */
};
typedef struct mie_gemm_args {
  const void* a;        /* bf16 */
  int64_t lda;          /* elements */
  const void* b;        /* bf16 */
  const void* b2;       /* bf16, MIE_GEMM_SWIGLU only */
  int64_t ldb;          /* elements, b and b2 */
  int64_t b_rows;       /* rows of b (and b2) over all groups */
  void* c;
  int64_t ldc;          /* elements */
  const float* resid;   /* MIE_GEMM_RESID */
  int64_t ldr;
  const int32_t* counts;  /* grouped: valid rows per group (device) or NULL */
  int M, N, K;
  int epilogue;
  int groups;
  int a_group_rows, b_group_rows, c_group_rows;
  int32_t* status;      /* optional device status word */
  const void* bias;     /* optional bf16 per-column bias (all but SwiGLU); group g
                           uses bias + g * bias_group_stride */
  int64_t bias_group_stride;
} mie_gemm_args;

/* Prefill per-token kernels (one warp per token; residual stream fp32, GEMM
 * operands bf16; weights bf16; hidden_dim a multiple of 32, at most 1024). */
typedef struct mie_prefill_norm_args {
  int tokens;
  int hidden_dim;
  int norm;                  /* MIE_NORM_RMS or MIE_NORM_LAYER */
  float eps;
  const int64_t* ids;        /* optional: first x[t] = embedding[ids[t]] (+ pos_embedding[pos0 + t]) */
  const void* embedding;     /* bf16 [vocab, hidden_dim] */
  const void* pos_embedding; /* bf16 [max_pos, hidden_dim] or NULL */
  int pos0;
  float* x;                  /* fp32 [tokens, hidden_dim] residual stream */
  const void* w;             /* bf16 norm weight */
  const void* b;             /* bf16 norm bias (LayerNorm) or NULL */
  void* out;                 /* bf16 [tokens, hidden_dim] */
} mie_prefill_norm_args;

typedef struct mie_prefill_rope_args {
  int tokens;
  int num_heads;
  int head_dim;
  int pos0;                  /* position of token 0 */
  const float* qkv;          /* fp32 [tokens, 3 * hidden]: q | k | v */
  const float* rope_cos;     /* fp32 [max_pos, head_dim / 2], or NULL (no RoPE) */
  const float* rope_sin;
  void* q_out;               /* bf16 [num_heads, tokens, head_dim] */
  void* k_out;
  void* v_out;
  void* k_cache;             /* bf16 cache of this layer */
  void* v_cache;
  const int32_t* block_table;  /* paged cache; NULL: contiguous (block_size = max positions) */
  int block_size;
  int64_t kv_stride_block;   /* elements */
  int64_t kv_stride_head;
  int64_t kv_stride_tok;
} mie_prefill_rope_args;

typedef struct mie_prefill_route_args {
  int tokens;
  int hidden_dim;
  int num_experts;           /* 2 .. 32, top-2 */
  int group_rows;            /* rows reserved per expert in `gathered` (>= tokens) */
  const void* x;             /* bf16 [tokens, hidden_dim], normalised: the rows gathered */
  const float* x_res;        /* fp32 [tokens, hidden_dim] residual stream; the router
                                reads norm(x_res) in fp32 */
  int norm;                  /* MIE_NORM_RMS or MIE_NORM_LAYER */
  float eps;
  const void* norm_w;        /* bf16 */
  const void* norm_b;        /* bf16 or NULL */
  const void* router_w;      /* bf16 [num_experts, hidden_dim] */
  float* logits;             /* optional fp32 [tokens, num_experts] */
  int32_t* counts;           /* [num_experts] rows per expert; zero on entry */
  float* weights;            /* [tokens, 2] softmax of the two selected logits */
  int32_t* ids_out;          /* [tokens, 2] selected experts (ties -> lower id) */
  int32_t* rows_out;         /* [tokens, 2] row of the token's copy in `gathered` */
  void* gathered;            /* bf16 [num_experts * group_rows, hidden_dim] */
} mie_prefill_route_args;

typedef struct mie_prefill_combine_args {
  int tokens;
  int hidden_dim;
  float* x;                  /* fp32 [tokens, hidden_dim], updated in place */
  const float* y;            /* fp32 expert outputs, rows as in rows[] */
  int64_t ldy;
  const float* weights;      /* [tokens, 2] */
  const int32_t* rows;       /* [tokens, 2] */
} mie_prefill_combine_args;

/* Causal self-attention of the prompt prefill (replaces the reference's
 * F.scaled_dot_product_attention(q, k, v, is_causal=True) of the prefill fast
 * path, src/moe_engine/model.py:252-256): o[t, h hd + d] = sum_{s <= t}
 * softmax_s(scale q_h[t] . k_h[s]) v_h[s][d], fp32 accumulation.  head_dim
 * 64 with 16-byte aligned q / k / v / out and ld_out a multiple of 8 runs on
 * the tensor cores (the probabilities rounded to bf16 for the P V product, as
 * flash attention does); other shapes on CUDA cores in fp32. */
typedef struct mie_prefill_attn_args {
  int tokens;
  int num_heads;
  int head_dim;              /* 64, 96 or 128 */
  float scale;               /* normally 1 / sqrt(head_dim) */
  const void* q;             /* bf16 [num_heads, tokens, head_dim] */
  const void* k;
  const void* v;
  void* out;                 /* bf16 [tokens, ld_out] */
  int64_t ld_out;            /* >= num_heads * head_dim */
  int32_t* status;           /* optional: MIE_ERR_TIMEOUT when a bounded wait of the
                                tensor-core kernel ran out (that launch wrote no rows) */
} mie_prefill_attn_args;

/* Expert-parallel all-reduce over peer memory.  No counterpart in the
 * reference (a single-GPU engine): it replaces the NCCL all-reduce of the
 * per-layer MoE partial in the expert-parallel decode (BASELINE config[4b]),
 *   out[i] = sum over ranks r = 0 .. world - 1, in rank order, of in_r[i].
 * Every rank writes its partial as tagged 64-bit words {f32 value, u32 call
 * number} into its slot of every rank's receive buffer (a peer's through a
 * CUDA IPC mapping, plain stores over NVLink) and polls its own buffer until
 * every rank's words carry this call's number; the sum order is the same on
 * every rank, so every rank holds the same bits.  The call number comes from
 * `seq` (device, zeroed once, advanced by each call), so the launch can be
 * captured in a CUDA graph.  All ranks make the same calls in the same order,
 * as with an NCCL collective.  Two buffer halves alternate by call number: a
 * rank cannot overwrite words a slower rank has yet to read. */
typedef struct mie_peer_reduce_args {
  int n;                     /* fp32 elements, 1 .. 1024 */
  int rank;
  int world;                 /* 1 .. MIE_PEER_MAX_RANKS */
  const float* in;           /* [n] this rank's partial */
  float* out;                /* [n] the sum (may be `in`) */
  uint64_t* bufs[MIE_PEER_MAX_RANKS];  /* every rank's receive buffer as this process maps it
                                          (its own at [rank]), mie_peer_buffer_bytes(n, world) each */
  uint32_t* seq;             /* this group's device call counter, zeroed once */
  int32_t* status;           /* optional: MIE_ERR_TIMEOUT when a rank's words did not arrive */
  int64_t wait_limit_ns;     /* 0: 200 ms */
} mie_peer_reduce_args;

/* Library management */
int mie_version(void);
int mie_init(int device);                 /* set kernel attributes; call before any capture */
const char* mie_status_string(int code);
const char* mie_last_cuda_error(void);   /* text of the last failed CUDA call on this thread, "" if none */
int mie_num_sms(int device);

/* Operators (see the table at the top of this file). */
int mie_moe_route(const mie_moe_args* a, void* stream);
int mie_moe_decode(const mie_moe_args* a, void* stream);
int mie_attn_decode(const mie_attn_args* a, void* stream);

/* mie_attn_decode_fixed_scratch -- no counterpart in the reference.
 *
 * The same attention decode as mie_attn_decode for callers that cannot
 * allocate device memory: a host runtime that owns all device memory and gives
 * its plugins no allocator, or a latency-critical caller that must not call
 * cudaMalloc / cudaFree (they can synchronise the device).  The caller passes
 * q, the cache and `out` as usual; a->partials, a->counters and a->max_splits
 * are ignored.  Split partials and merge counters live in one fixed array
 * inside libmie.so: 64 counter words + 65,536 floats (256 KB), which every GPU
 * that loads the library holds until the process exits.  Limits: num_heads <=
 * 64 and num_heads * splits * (head_dim + 2) <= 65,536; larger requests return
 * MIE_ERR_SCRATCH_LIMIT and launch nothing; a->defer_merge must be 0 (the
 * partials would stay in the library's array, where no consumer can read them:
 * MIE_ERR_INVALID).  The request is validated before the size limit is checked,
 * so a malformed request returns MIE_ERR_INVALID / MIE_ERR_UNSUPPORTED as with
 * mie_attn_decode.  Nothing is allocated: no cudaMalloc, cudaFree or allocating
 * library call.  The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress, with that device current) and zeroes its counters with
 * cudaMemsetAsync on the caller's stream, so make the first call on each device
 * before any stream capture.  All calls share the
 * array and each call returns the counters to zero: calls that overlap on
 * the GPU (for example on two streams at once) race and corrupt each other. */
int mie_attn_decode_fixed_scratch(const mie_attn_args* a, void* stream);
int mie_qkv_rope_store(const mie_qkv_args* a, void* stream);
int mie_proj_residual(const mie_proj_args* a, void* stream);
int mie_lmhead_argmax(const mie_lmhead_args* a, void* stream);

/* Whole-step launchers.  mie_decode_layer / mie_decode_head let a caller put a
 * collective between a layer's MoE and the next consumer (expert parallel).
 * mie_decode_step runs the persistent single-launch step when d->step_scratch
 * is set (MIE_ERR_UNSUPPORTED when the shapes have no persistent kernel), else
 * the per-op launch sequence. */
int mie_decode_step(const mie_step_desc* d, void* stream);
/* Bytes of d->step_scratch the persistent step needs for this description on
 * the current device (> 0), or -status when the persistent step does not
 * support it (hidden_dim and expert_hidden_dim <= 768, head_dim <= 128, no
 * expert parallelism, num_layers <= 48).  Launches nothing. */
int64_t mie_step_scratch_bytes(const mie_step_desc* d);
/* Which persistent kernel mie_decode_step would run for this description on
 * the current device: MIE_STEP_CLUSTER (clusters of 6 CTAs; bf16, head_dim
 * 64, RMSNorm, RoPE, SwiGLU, no biases, greedy) or MIE_STEP_FLAT (one CTA per
 * SM; every other supported shape), or -status.  Launches nothing.  No
 * counterpart in the reference (its decode step is a sequence of Python-level
 * ops, src/moe_engine/model.py:543-565). */
int mie_step_kernel_of(const mie_step_desc* d);
int mie_decode_layer(const mie_step_desc* d, int layer, void* stream);
int mie_decode_head(const mie_step_desc* d, void* stream);

/* Prefill GEMM (see mie_gemm_args) and per-token kernels. */
int mie_gemm(const mie_gemm_args* a, void* stream);
int mie_prefill_norm(const mie_prefill_norm_args* a, void* stream);
int mie_prefill_rope_kv(const mie_prefill_rope_args* a, void* stream);
int mie_prefill_route(const mie_prefill_route_args* a, void* stream);
int mie_prefill_combine(const mie_prefill_combine_args* a, void* stream);
int mie_prefill_attention(const mie_prefill_attn_args* a, void* stream);

/* Expert-parallel all-reduce over peer memory (see mie_peer_reduce_args) and
 * the CUDA IPC plumbing of its receive buffers; the caller exchanges the
 * 64-byte handles between its processes (e.g. torch.distributed). */
int64_t mie_peer_buffer_bytes(int n, int world);
int mie_peer_reduce(const mie_peer_reduce_args* a, void* stream);
int mie_peer_alloc(int64_t bytes, void** ptr);         /* zeroed device memory, its own allocation */
int mie_peer_free(void* ptr);
int mie_peer_handle(const void* ptr, void* handle64);  /* cudaIpcGetMemHandle of an mie_peer_alloc buffer */
int mie_peer_open(const void* handle64, void** ptr);   /* cudaIpcOpenMemHandle (another process's buffer) */
int mie_peer_close(void* ptr);

#ifdef __cplusplus
}
#endif
#endif /* MIE_H */
