// Batch-one GEMV kernels of the decode step, sm_100a:
//
//  * qkv_kernel      norm(x) -> QKV GEMV [3D, D] -> RoPE(q, k) -> q to scratch,
//                    k / v into the cache slot of the device position
//                    (reference: src/moe_engine/model.py:226-234,247,495,557-558;
//                    the paged slot math of model.py:145-147,167-178).
//  * proj_kernel     out += W in + b (out_proj + residual, model.py:268-269,495),
//                    optionally merging split-K attention partials into `in`.
//  * lmhead_kernel   final norm -> tied LM head [V, D] -> argmax (ties -> lower
//                    id) + the step's device bookkeeping (model.py:562-565,
//                    600-603,615).
//
// A warp owns whole weight rows and loads them straight into registers
// (stream.cuh).  Rows are static, so each warp's first rows are requested
// BEFORE griddepcontrol.wait: under programmatic dependent launch the weight
// fetch overlaps the previous kernel.  The LM head keeps the next batch of
// rows in flight while it reduces the current one.
#include <utility>

#include "kernels.h"
#include "stream.cuh"

namespace mie {

namespace {

// Attention merge in proj_kernel: heads x splits weights in static shared memory.
constexpr int kMaxMergeHeads = 64;
constexpr int kMaxMergeSplits = 64;

__device__ __forceinline__ const uint4* row_ptr(const void* base, int64_t row, int64_t row_bytes) {
  return reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(base) + row * row_bytes);
}

// ---------------------------------------------------------------------------
// QKV
// ---------------------------------------------------------------------------
// Work unit = one RoPE pair of one head of one section (q, k or v): rows
// (h*hd + i) and (h*hd + i + hd/2) of that section, i < hd/2.  A CTA owns a
// contiguous unit range; warp w takes units u0 + w, u0 + w + nwarps, ...
// Both rows of a unit are reduced by the same warp, so lane 0 applies RoPE and
// stores without any exchange.
template <typename W>
__global__ void __launch_bounds__(512) qkv_kernel(const mie_qkv_args a, GemvLayout L) {
  extern __shared__ __align__(16) float xs[];  // [D]
  __shared__ float red[16];
  __shared__ int pos_s;
  __shared__ int64_t slot_off_s, tok_s;
  constexpr int PV = Elem<W>::kPerVec;
  const int D = a.hidden_dim, H = a.num_heads, hd = a.head_dim, half = hd / 2;
  const int U = 3 * H * half;
  const int G = gridDim.x, c = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int NW = blockDim.x >> 5;
  int u0, u1;
  split_range(U, c, G, &u0, &u1);
  const int nu = u1 - u0;
  const int nvec = D / PV;
  const int64_t row_bytes = (int64_t)D * sizeof(W);
  const bool one_seg = nvec <= Seg<W>::kVecs;
  auto unit_rows = [&](int u, int64_t* ra) {
    const int grp = u / half, i = u - grp * half, sec = grp / H, h = grp - sec * H;
    *ra = (int64_t)sec * D + (int64_t)h * hd + i;
  };

  // First unit of this warp: both rows requested before the PDL wait.
  RowRegs<W> wa, wb;
  if (one_seg && warp < nu) {
    int64_t ra;
    unit_rows(u0 + warp, &ra);
    row_load<W>(wa, row_ptr(a.w, ra, row_bytes), nvec, 0);
    row_load<W>(wb, row_ptr(a.w, ra + half, row_bytes), nvec, 0);
  }

  pdl_wait();
  if (skip_requested(a.skip)) {
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
    if (a.embedding) {
      int64_t t = __ldcg(a.token);
      if (t < 0 || t >= a.vocab) {
        set_status(a.status, MIE_ERR_RANGE);
        t = 0;
      }
      tok_s = t;
    }
  }
  __syncthreads();
  const int pos = pos_s;

  // input vector: x, or the token embedding (+ learned position) for layer 0
  if (a.embedding) {
    const int64_t tok = tok_s;
    for (int i = tid; i < D; i += blockDim.x) {
      float v = load_any(a.embedding, a.dtype, tok * D + i);
      if (a.pos_embedding) v += load_any(a.pos_embedding, a.dtype, (int64_t)pos * D + i);
      xs[i] = v;
      if (c == 0) a.x[i] = v;  // the residual stream starts at the embedding
    }
    load_and_norm(xs, nullptr, MIE_F32, nullptr, D, a.norm, a.eps, a.norm_w, a.norm_b, a.dtype, red);
  } else {
    load_and_norm(xs, a.x, MIE_F32, a.x_add, D, a.norm, a.eps, a.norm_w, a.norm_b, a.dtype, red);
  }
  float xr[Seg<W>::kNV * PV];
  load_x_regs<W>(xr, xs, nvec);

  const int64_t slot_off = slot_off_s;
  for (int k = warp; k < nu; k += NW) {
    const int u = u0 + k;
    int64_t ra;
    unit_rows(u, &ra);
    float x1, x2;
    if (one_seg) {
      if (k != warp) {
        row_load<W>(wa, row_ptr(a.w, ra, row_bytes), nvec, 0);
        row_load<W>(wb, row_ptr(a.w, ra + half, row_bytes), nvec, 0);
      }
      x1 = warp_sum(row_dot_regs<W>(wa, xr));
      x2 = warp_sum(row_dot_regs<W>(wb, xr));
    } else {
      x1 = warp_row_dot<W>(row_ptr(a.w, ra, row_bytes), nvec, xs);
      x2 = warp_row_dot<W>(row_ptr(a.w, ra + half, row_bytes), nvec, xs);
    }
    if (lane == 0) {
      const int grp = u / half, i = u - grp * half, sec = grp / H, h = grp - sec * H;
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
}

// ---------------------------------------------------------------------------
// out_proj (+ residual): out[r] = (acc ? out[r] : 0) + add[r] + W[r].in + b[r]
// ---------------------------------------------------------------------------
template <typename W>
__global__ void __launch_bounds__(256) proj_kernel(const mie_proj_args a, GemvLayout L) {
  extern __shared__ __align__(16) float xs[];  // [cols]
  __shared__ float w_s[kMaxMergeHeads * kMaxMergeSplits];
  constexpr int PV = Elem<W>::kPerVec;
  const int G = gridDim.x, c = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int NW = blockDim.x >> 5;
  int r0, r1;
  split_range(a.rows, c, G, &r0, &r1);
  const int nr = r1 - r0;
  const int nvec = a.cols / PV;
  const int64_t row_bytes = (int64_t)a.cols * sizeof(W);
  const bool one_seg = nvec <= Seg<W>::kVecs;

  RowRegs<W> wr;
  if (one_seg && warp < nr) row_load<W>(wr, row_ptr(a.w, r0 + warp, row_bytes), nvec, 0);

  pdl_wait();
  if (skip_requested(a.skip)) {
    pdl_trigger();
    return;
  }
  pdl_trigger();
  if (a.attn_partials) {
    // Input = attention output, merged here from the split-K partials
    // (m, l, acc[hd]) of every head: o = sum_s acc_s e^(m_s - M) / sum_s l_s e^(m_s - M).
    const int H = a.attn_heads, hd = a.attn_head_dim, Sp = a.attn_splits;
    auto part = [&](int h, int s) { return a.attn_partials + ((size_t)h * a.attn_max_splits + s) * (hd + 2); };
    for (int h = warp; h < H; h += NW) {
      float m[2], l[2];
      for (int k = 0; k < 2; ++k) {
        const int s = lane + 32 * k;
        m[k] = s < Sp ? __ldcg(part(h, s)) : -INFINITY;
        l[k] = s < Sp ? __ldcg(part(h, s) + 1) : 0.f;
      }
      const float M = warp_max(fmaxf(m[0], m[1]));
      float e[2];
      for (int k = 0; k < 2; ++k) e[k] = m[k] == -INFINITY ? 0.f : expf(m[k] - M);
      const float Lsum = warp_sum(l[0] * e[0] + l[1] * e[1]);
      for (int k = 0; k < 2; ++k) {
        const int s = lane + 32 * k;
        if (s < Sp) w_s[h * kMaxMergeSplits + s] = e[k] / Lsum;
      }
    }
    __syncthreads();
    for (int i = tid; i < H * hd; i += blockDim.x) {
      const int h = i / hd, d = i - h * hd;
      float o = 0.f;
      for (int s = 0; s < Sp; ++s) o = fmaf(w_s[h * kMaxMergeSplits + s], __ldcg(part(h, s) + 2 + d), o);
      xs[i] = o;
    }
  } else {
    for (int i = tid; i < a.cols; i += blockDim.x) xs[i] = __ldcg(a.in + i);
  }
  __syncthreads();
  float xr[Seg<W>::kNV * PV];
  if (one_seg) load_x_regs<W>(xr, xs, nvec);

  for (int k = warp; k < nr; k += NW) {
    const int r = r0 + k;
    float y;
    if (one_seg) {
      if (k != warp) row_load<W>(wr, row_ptr(a.w, r, row_bytes), nvec, 0);
      y = warp_sum(row_dot_regs<W>(wr, xr));
    } else {
      y = warp_row_dot<W>(row_ptr(a.w, r, row_bytes), nvec, xs);
    }
    if (lane == 0) {
      if (a.b) y += load_any(a.b, a.dtype, r);
      if (a.add) y += __ldcg(a.add + r);
      if (a.accumulate) y += __ldcg(a.out + r);
      a.out[r] = y;
    }
  }
}

// ---------------------------------------------------------------------------
// LM head + argmax
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

// Rows per batch per warp: the next batch's loads are in flight while the
// current one is reduced (2 x 6 16-byte vectors per lane either way).
template <typename W>
struct LmBatch {
  static constexpr int kRows = sizeof(W) == 2 ? 2 : 1;
};

template <typename W>
__global__ void __launch_bounds__(512) lmhead_kernel(const mie_lmhead_args a, GemvLayout L) {
  extern __shared__ __align__(16) float xs[];  // [D]
  __shared__ float red[16];
  __shared__ float wbest_v[16];
  __shared__ int wbest_i[16];
  __shared__ int last_s;
  constexpr int PV = Elem<W>::kPerVec;
  constexpr int RB = LmBatch<W>::kRows;
  const int D = a.hidden_dim;
  const int G = gridDim.x, c = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int NW = blockDim.x >> 5;
  int r0, r1;
  split_range(a.vocab, c, G, &r0, &r1);
  const int nvec = D / PV;
  const int64_t row_bytes = (int64_t)D * sizeof(W);
  const bool one_seg = nvec <= Seg<W>::kVecs;
  // this warp's rows: r0 + warp + NW * k, k < nmine (ascending)
  const int nmine = (r1 - r0 - warp + NW - 1) / NW > 0 ? (r1 - r0 - warp + NW - 1) / NW : 0;
  auto row_of = [&](int k) { return r0 + warp + NW * k; };

  RowRegs<W> cur[RB], nxt[RB];
  if (one_seg) {
#pragma unroll
    for (int r = 0; r < RB; ++r)
      if (r < nmine) row_load<W>(cur[r], row_ptr(a.w, row_of(r), row_bytes), nvec, 0);
  }

  pdl_wait();
  if (skip_requested(a.skip)) {
    pdl_trigger();
    return;
  }
  pdl_trigger();
  load_and_norm(xs, a.x, MIE_F32, a.x_add, D, a.norm, a.eps, a.norm_w, a.norm_b, a.dtype, red);

  float best_v = -INFINITY;  // per warp, valid on lane 0
  int best_i = 0x7fffffff;
  auto emit = [&](int row, float v) {
    if (a.b) v += load_any(a.b, a.dtype, row);
    if (a.logits) a.logits[row] = v;
    if (better(v, row, best_v, best_i)) {
      best_v = v;
      best_i = row;
    }
  };
  if (one_seg) {
    float xr[Seg<W>::kNV * PV];
    load_x_regs<W>(xr, xs, nvec);
    for (int kb = 0; kb < nmine; kb += RB) {
#pragma unroll
      for (int r = 0; r < RB; ++r)
        if (kb + RB + r < nmine) row_load<W>(nxt[r], row_ptr(a.w, row_of(kb + RB + r), row_bytes), nvec, 0);
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        if (kb + r < nmine) {
          const float v = warp_sum(row_dot_regs<W>(cur[r], xr));
          if (lane == 0) emit(row_of(kb + r), v);
        }
      }
#pragma unroll
      for (int r = 0; r < RB; ++r) cur[r] = nxt[r];
    }
  } else {
    for (int k = 0; k < nmine; ++k) {
      const float v = warp_row_dot<W>(row_ptr(a.w, row_of(k), row_bytes), nvec, xs);
      if (lane == 0) emit(row_of(k), v);
    }
  }

  if (lane == 0) {
    wbest_v[warp] = best_v;
    wbest_i[warp] = best_i;
  }
  __syncthreads();
  if (tid == 0) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int w = 0; w < NW; ++w)
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
    const int k = __ldcg(a.log_count);
    if (k < a.log_capacity) a.tokens_log[k] = bi;
    *a.log_count = k + 1;
  }
  if (a.done && bi == a.eos_id) *a.done = 1;
  __threadfence();
  *a.counter = 0u;
}

GemvLayout vec_layout(int vec_len) {
  GemvLayout L{};
  L.smem = (uint32_t)(sizeof(float) * ((vec_len + 3) & ~3));
  return L;
}

}  // namespace

GemvLayout qkv_layout(const mie_qkv_args& a, int) { return vec_layout(a.hidden_dim); }
int qkv_launch(const mie_qkv_args& a, const GemvLayout& L, int grid, cudaStream_t st, bool pdl) {
  auto k = a.dtype == MIE_BF16 ? qkv_kernel<__nv_bfloat16> : qkv_kernel<float>;
  return launch(k, dim3(grid), dim3(512), L.smem, st, pdl, a, L);
}

GemvLayout proj_layout(const mie_proj_args& a, int) { return vec_layout(a.cols); }
int proj_launch(const mie_proj_args& a, const GemvLayout& L, int grid, cudaStream_t st, bool pdl) {
  auto k = a.dtype == MIE_BF16 ? proj_kernel<__nv_bfloat16> : proj_kernel<float>;
  return launch(k, dim3(grid), dim3(256), L.smem, st, pdl, a, L);
}

GemvLayout lmhead_layout(const mie_lmhead_args& a, int) { return vec_layout(a.hidden_dim); }
int lmhead_launch(const mie_lmhead_args& a, const GemvLayout& L, int grid, cudaStream_t st, bool pdl) {
  auto k = a.dtype == MIE_BF16 ? lmhead_kernel<__nv_bfloat16> : lmhead_kernel<float>;
  return launch(k, dim3(grid), dim3(512), L.smem, st, pdl, a, L);
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
