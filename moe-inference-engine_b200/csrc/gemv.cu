// Batch-one GEMV kernels of the decode step, sm_100a:
//
//  * qkv_kernel      norm(x) -> QKV GEMV [3D, D] -> RoPE(q, k) -> q to scratch,
//                    k / v into the cache slot of the device position
//                    (reference: src/moe_engine/model.py:226-234,247,495,557-558;
//                    the paged slot math of model.py:145-147,167-178).
//  * proj_kernel     out += W in + b (out_proj + residual, model.py:268-269,495).
//  * lmhead_kernel   final norm -> tied LM head [V, D] -> argmax (ties -> lower
//                    id) + the step's device bookkeeping (model.py:562-565,
//                    600-603,615).
//
// All three stream their weight rows with the TMA bulk ring of stream.cuh.
// Weights do not depend on the producer grid, so the first ring slots are
// filled BEFORE griddepcontrol.wait: under programmatic dependent launch the
// weight fetch overlaps the previous kernel.
#include <utility>

#include "kernels.h"
#include "stream.cuh"

namespace mie {

namespace {

constexpr int kMaxChunks = 160;
constexpr int kThreads = 256;

struct GemvSmem {
  Ring R;
  float* xs;
  float* res;
  Chunk* chunks;
};

__device__ __forceinline__ GemvSmem gemv_smem(uint8_t* smem, const GemvLayout& L) {
  GemvSmem g;
  g.R.bar = reinterpret_cast<uint64_t*>(smem + L.off_bar);
  g.R.data = smem + L.off_ring;
  g.R.nslot = L.nslot;
  g.R.slot_bytes = L.slot_bytes;
  g.xs = reinterpret_cast<float*>(smem + L.off_x);
  g.res = reinterpret_cast<float*>(smem + L.off_res);
  g.chunks = reinterpret_cast<Chunk*>(smem + L.off_chunks);
  return g;
}

// ---------------------------------------------------------------------------
// QKV
// ---------------------------------------------------------------------------
// Work unit = one RoPE pair of one head of one section (q, k or v): rows
// (h*hd + i) and (h*hd + i + hd/2) of that section, i < hd/2.  A CTA owns a
// contiguous unit range, i.e. for each (section, head) it touches two
// contiguous row runs, so no weight repacking is needed.
enum : uint8_t { kTagFirstHalf = 0, kTagSecondHalf = 1 };

template <typename W>
__global__ void __launch_bounds__(kThreads) qkv_kernel(const mie_qkv_args a, GemvLayout L) {
  extern __shared__ __align__(128) uint8_t smem[];
  GemvSmem S = gemv_smem(smem, L);
  __shared__ float red[kThreads / 32];
  __shared__ int n_s;
  __shared__ int pos_s;
  __shared__ int64_t slot_off_s;
  const int D = a.hidden_dim, H = a.num_heads, hd = a.head_dim, half = hd / 2;
  const int U = 3 * H * half;
  const int G = gridDim.x, c = blockIdx.x, tid = threadIdx.x;
  int u0, u1;
  split_range(U, c, G, &u0, &u1);
  const int nu = u1 - u0;
  float* resA = S.res;
  float* resB = S.res + L.max_units;
  const uint64_t pol = policy_evict_first();
  const uint32_t row_bytes = (uint32_t)(D * sizeof(W));
  const int cap = (int)(L.slot_bytes / row_bytes);

  if (tid == 0) {
    ring_init(S.R);
    int n = 0;
    bool ok = true;
    for (int u = u0; u < u1;) {
      const int grp = u / half, i0 = u - grp * half;
      const int i1 = min(half, i0 + (u1 - u));
      const int sec = grp / H, h = grp - sec * H;
      const int64_t base = (int64_t)sec * D + (int64_t)h * hd;
      ok &= push_rows(S.chunks, &n, kMaxChunks, a.w, base + i0, i1 - i0, row_bytes, cap, kTagFirstHalf, 0, u - u0);
      ok &= push_rows(S.chunks, &n, kMaxChunks, a.w, base + half + i0, i1 - i0, row_bytes, cap, kTagSecondHalf, 0,
                      u - u0);
      u += i1 - i0;
    }
    if (!ok) {
      set_status(a.status, MIE_ERR_INVALID);
      n = 0;
    }
    n_s = n;
    for (int i = 0; i < min(n, S.R.nslot); ++i) ring_issue(S.R, S.chunks[i], i, pol);
  }
  __syncthreads();
  const int n = n_s;

  pdl_wait();
  if (skip_requested(a.skip)) {
    if (tid == 0) ring_drain(S.R, 0, min(n, S.R.nslot), a.status);
    __syncthreads();
    pdl_trigger();
    return;
  }
  pdl_trigger();

  // position + cache slot of the new token
  if (tid == 0) {
    int p = __ldcg(a.pos);
    if (p < 0 || p >= a.max_pos) {
      set_status(a.status, MIE_ERR_RANGE);
      p = 0;
    }
    int64_t blk = p / a.block_size;
    if (a.block_table) {
      int pb = __ldcg(a.block_table + blk);
      if (pb < 0 || pb >= a.num_blocks) {
        set_status(a.status, MIE_ERR_RANGE);
        pb = 0;
      }
      blk = pb;
    }
    pos_s = p;
    slot_off_s = blk * a.stride_block + (int64_t)(p % a.block_size) * a.stride_tok;
  }
  __syncthreads();
  const int pos = pos_s;

  // input vector: x, or the token embedding (+ learned position) for layer 0
  if (a.embedding) {
    __shared__ int64_t tok_s;
    if (tid == 0) {
      int64_t t = __ldcg(a.token);
      if (t < 0 || t >= a.vocab) {
        set_status(a.status, MIE_ERR_RANGE);
        t = 0;
      }
      tok_s = t;
    }
    __syncthreads();
    const int64_t tok = tok_s;
    for (int i = tid; i < D; i += blockDim.x) {
      float v = load_any(a.embedding, a.dtype, tok * D + i);
      if (a.pos_embedding) v += load_any(a.pos_embedding, a.dtype, (int64_t)pos * D + i);
      S.xs[i] = v;
      if (c == 0) a.x[i] = v;  // residual stream starts at the embedding
    }
    __syncthreads();
    load_and_norm(S.xs, S.xs, MIE_F32, nullptr, D, a.norm, a.eps, a.norm_w, a.norm_b, a.dtype, red);
  } else {
    load_and_norm(S.xs, a.x, MIE_F32, a.x_add, D, a.norm, a.eps, a.norm_w, a.norm_b, a.dtype, red);
  }

  const bool ok = ring_consume(S.R, S.chunks, n, min(n, S.R.nslot), pol, a.status,
                               [&](int, const Chunk& ch, const uint8_t* s) {
                                 float* dst = ch.tag == kTagFirstHalf ? resA : resB;
                                 chunk_dot_rows<W>(s, ch.rows, D, S.xs, [&](int r, float v) { dst[ch.out + r] = v; });
                               });
  if (!ok) return;

  // epilogue: bias, RoPE on q / k, stores
  const int64_t slot_off = slot_off_s;
  for (int k = tid; k < nu; k += blockDim.x) {
    const int u = u0 + k, grp = u / half, i = u - grp * half;
    const int sec = grp / H, h = grp - sec * H;
    const int64_t ra = (int64_t)sec * D + (int64_t)h * hd + i;
    float x1 = resA[k], x2 = resB[k];
    if (a.b) {
      x1 += load_any(a.b, a.dtype, ra);
      x2 += load_any(a.b, a.dtype, ra + half);
    }
    if (sec < 2 && a.rope_cos) {
      const float cs = a.rope_cos[(int64_t)pos * half + i], sn = a.rope_sin[(int64_t)pos * half + i];
      const float y1 = x1 * cs - x2 * sn;
      const float y2 = x2 * cs + x1 * sn;
      x1 = y1;
      x2 = y2;
    }
    if (sec == 0) {
      a.q_out[h * hd + i] = x1;
      a.q_out[h * hd + i + half] = x2;
    } else {
      void* cache = sec == 1 ? a.k_cache : a.v_cache;
      const int64_t o = slot_off + (int64_t)h * a.stride_head;
      store_any(cache, a.kv_dtype, o + i, x1);
      store_any(cache, a.kv_dtype, o + i + half, x2);
    }
  }
}

// ---------------------------------------------------------------------------
// out_proj (+ residual): out[r] = (acc ? out[r] : 0) + add[r] + W[r].in + b[r]
// ---------------------------------------------------------------------------
template <typename W>
__global__ void __launch_bounds__(kThreads) proj_kernel(const mie_proj_args a, GemvLayout L) {
  extern __shared__ __align__(128) uint8_t smem[];
  GemvSmem S = gemv_smem(smem, L);
  __shared__ int n_s;
  const int G = gridDim.x, c = blockIdx.x, tid = threadIdx.x;
  int r0, r1;
  split_range(a.rows, c, G, &r0, &r1);
  const uint64_t pol = policy_evict_first();
  const uint32_t row_bytes = (uint32_t)(a.cols * sizeof(W));
  const int cap = (int)(L.slot_bytes / row_bytes);
  if (tid == 0) {
    ring_init(S.R);
    int n = 0;
    if (!push_rows(S.chunks, &n, kMaxChunks, a.w, r0, r1 - r0, row_bytes, cap, 0, 0, 0)) {
      set_status(a.status, MIE_ERR_INVALID);
      n = 0;
    }
    n_s = n;
    for (int i = 0; i < min(n, S.R.nslot); ++i) ring_issue(S.R, S.chunks[i], i, pol);
  }
  __syncthreads();
  const int n = n_s;
  pdl_wait();
  if (skip_requested(a.skip)) {
    if (tid == 0) ring_drain(S.R, 0, min(n, S.R.nslot), a.status);
    __syncthreads();
    pdl_trigger();
    return;
  }
  pdl_trigger();
  for (int i = tid; i < a.cols; i += blockDim.x) S.xs[i] = a.in[i];
  __syncthreads();
  const bool ok = ring_consume(S.R, S.chunks, n, min(n, S.R.nslot), pol, a.status,
                               [&](int, const Chunk& ch, const uint8_t* s) {
                                 chunk_dot_rows<W>(s, ch.rows, a.cols, S.xs,
                                                   [&](int r, float v) { S.res[ch.out + r] = v; });
                               });
  if (!ok) return;
  for (int k = tid; k < r1 - r0; k += blockDim.x) {
    const int r = r0 + k;
    float y = S.res[k];
    if (a.b) y += load_any(a.b, a.dtype, r);
    if (a.add) y += a.add[r];
    if (a.accumulate) y += a.out[r];
    a.out[r] = y;
  }
}

// ---------------------------------------------------------------------------
// LM head + argmax
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

template <typename W>
__global__ void __launch_bounds__(kThreads) lmhead_kernel(const mie_lmhead_args a, GemvLayout L) {
  extern __shared__ __align__(128) uint8_t smem[];
  GemvSmem S = gemv_smem(smem, L);
  __shared__ float red[kThreads / 32];
  __shared__ float wbest_v[kThreads / 32];
  __shared__ int wbest_i[kThreads / 32];
  __shared__ int n_s, last_s;
  const int D = a.hidden_dim;
  const int G = gridDim.x, c = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int r0, r1;
  split_range(a.vocab, c, G, &r0, &r1);
  const uint64_t pol = policy_evict_first();
  const uint32_t row_bytes = (uint32_t)(D * sizeof(W));
  const int cap = (int)(L.slot_bytes / row_bytes);
  if (tid == 0) {
    ring_init(S.R);
    int n = 0;
    if (!push_rows(S.chunks, &n, kMaxChunks, a.w, r0, r1 - r0, row_bytes, cap, 0, 0, r0)) {
      set_status(a.status, MIE_ERR_INVALID);
      n = 0;
    }
    n_s = n;
    for (int i = 0; i < min(n, S.R.nslot); ++i) ring_issue(S.R, S.chunks[i], i, pol);
  }
  __syncthreads();
  const int n = n_s;
  pdl_wait();
  if (skip_requested(a.skip)) {
    if (tid == 0) ring_drain(S.R, 0, min(n, S.R.nslot), a.status);
    __syncthreads();
    pdl_trigger();
    return;
  }
  pdl_trigger();
  load_and_norm(S.xs, a.x, MIE_F32, a.x_add, D, a.norm, a.eps, a.norm_w, a.norm_b, a.dtype, red);

  float best_v = -INFINITY;  // per warp, valid on lane 0
  int best_i = 0x7fffffff;
  const bool ok = ring_consume(S.R, S.chunks, n, min(n, S.R.nslot), pol, a.status,
                               [&](int, const Chunk& ch, const uint8_t* s) {
                                 chunk_dot_rows<W>(s, ch.rows, D, S.xs, [&](int r, float v) {
                                   const int row = ch.out + r;
                                   if (a.b) v += load_any(a.b, a.dtype, row);
                                   if (a.logits) a.logits[row] = v;
                                   if (better(v, row, best_v, best_i)) {
                                     best_v = v;
                                     best_i = row;
                                   }
                                 });
                               });
  if (!ok) return;
  if (lane == 0) {
    wbest_v[warp] = best_v;
    wbest_i[warp] = best_i;
  }
  __syncthreads();
  if (tid == 0) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w)
      if (better(wbest_v[w], wbest_i[w], bv, bi)) {
        bv = wbest_v[w];
        bi = wbest_i[w];
      }
    a.partial_val[c] = bv;
    a.partial_idx[c] = bi;
    __threadfence();
    last_s = atom_add_acq_rel_gpu(a.counter, 1u) == (uint32_t)(G - 1);
  }
  __syncthreads();
  if (!last_s || tid != 0) return;
  __threadfence();
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int j = 0; j < G; ++j) {
    const float v = __ldcg(a.partial_val + j);
    const int i = __ldcg(a.partial_idx + j);
    if (better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
  if (bi < 0 || bi >= a.vocab) {  // every logit NaN
    set_status(a.status, MIE_ERR_RANGE);
    bi = 0;
  }
  if (a.token_out) *a.token_out = bi;
  if (a.pos) *a.pos = __ldcg(a.pos) + 1;
  if (a.tokens_log && a.log_count) {
    const int k = *a.log_count;
    if (k < a.log_capacity) a.tokens_log[k] = bi;
    *a.log_count = k + 1;
  }
  if (a.done && bi == a.eos_id) *a.done = 1;
  __threadfence();
  *a.counter = 0u;
}

size_t align128(size_t v) { return (v + 127) & ~size_t(127); }

GemvLayout gemv_layout(int units_per_cta_max, int vec_len, int slot_bytes, int nslot, int res_arrays) {
  GemvLayout L{};
  L.nslot = nslot;
  L.slot_bytes = (uint32_t)slot_bytes;
  L.max_units = units_per_cta_max;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    off = align128(off);
    const size_t at = off;
    off += bytes;
    return (uint32_t)at;
  };
  L.off_bar = take(sizeof(uint64_t) * nslot);
  L.off_ring = take((size_t)nslot * slot_bytes);
  L.off_x = take(sizeof(float) * vec_len);
  L.off_res = take(sizeof(float) * (size_t)res_arrays * units_per_cta_max);
  L.off_chunks = take(sizeof(Chunk) * kMaxChunks);
  L.smem = (uint32_t)align128(off);
  return L;
}

}  // namespace

GemvLayout qkv_layout(const mie_qkv_args& a, int grid) {
  const int U = 3 * a.num_heads * (a.head_dim / 2);
  return gemv_layout((U + grid - 1) / grid + 1, a.hidden_dim, 16 * 1024, 4, 2);
}
int qkv_launch(const mie_qkv_args& a, const GemvLayout& L, int grid, cudaStream_t st, bool pdl) {
  auto k = a.dtype == MIE_BF16 ? qkv_kernel<__nv_bfloat16> : qkv_kernel<float>;
  return launch(k, dim3(grid), dim3(kThreads), L.smem, st, pdl, a, L);
}

GemvLayout proj_layout(const mie_proj_args& a, int grid) {
  return gemv_layout((a.rows + grid - 1) / grid + 1, a.cols, 16 * 1024, 2, 1);
}
int proj_launch(const mie_proj_args& a, const GemvLayout& L, int grid, cudaStream_t st, bool pdl) {
  auto k = a.dtype == MIE_BF16 ? proj_kernel<__nv_bfloat16> : proj_kernel<float>;
  return launch(k, dim3(grid), dim3(kThreads), L.smem, st, pdl, a, L);
}

GemvLayout lmhead_layout(const mie_lmhead_args& a, int grid) {
  return gemv_layout(1, a.hidden_dim, 16 * 1024, 6, 1);
}
int lmhead_launch(const mie_lmhead_args& a, const GemvLayout& L, int grid, cudaStream_t st, bool pdl) {
  auto k = a.dtype == MIE_BF16 ? lmhead_kernel<__nv_bfloat16> : lmhead_kernel<float>;
  return launch(k, dim3(grid), dim3(kThreads), L.smem, st, pdl, a, L);
}

void gemv_set_attributes() {
  set_max_smem(qkv_kernel<__nv_bfloat16>);
  set_max_smem(qkv_kernel<float>);
  set_max_smem(proj_kernel<__nv_bfloat16>);
  set_max_smem(proj_kernel<float>);
  set_max_smem(lmhead_kernel<__nv_bfloat16>);
  set_max_smem(lmhead_kernel<float>);
}

}  // namespace mie
