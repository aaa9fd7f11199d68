// Prompt prefill: the per-token kernels around the tensor-core GEMMs
// (csrc/gemm.cu).  One warp per token everywhere; the residual stream x stays
// fp32, GEMM operands are bf16.
//
//   prefill_norm      x[t] = embedding[id] (+ learned position) when ids are
//                     given; out[t] = norm(x[t]) as bf16        (model.py:491-492,557-558)
//   prefill_rope_kv   q / k / v rows of the QKV GEMM -> RoPE on q and k ->
//                     [H, T, hd] bf16 operands for the attention and the K/V
//                     cache slots of positions pos0 + t (paged through the
//                     block table, or contiguous)             (model.py:226-247)
//   prefill_route     router logits (fp32, from the fp32 residual normalised
//                     again here), top-2 with ties to the lower id,
//                     softmax of the two logits; each token's row is copied to
//                     the next free row of both selected experts' groups
//                     (counts[e] grows by atomics: the order of the rows in a
//                     group varies, each row's result does not)  (model.py:443-452)
//   prefill_combine   x[t] += w0 y[row0] + w1 y[row1] in that order (model.py:453-461)
#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace mie {
namespace {

constexpr int kPfThreads = 256;  // 8 warps, one token each
constexpr int kPfWarps = kPfThreads / 32;
constexpr int kPfMaxDim = 1024;  // hidden_dim: at most 32 elements per lane

__device__ __forceinline__ float bf(const __nv_bfloat16* p, int64_t i) { return __bfloat162float(p[i]); }

__global__ void __launch_bounds__(kPfThreads) prefill_norm_kernel(const mie_prefill_norm_args a) {
  const int t = blockIdx.x * kPfWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (t >= a.tokens) return;
  const int D = a.hidden_dim;
  float* xr = a.x + (int64_t)t * D;
  constexpr int kPer = kPfMaxDim / 32;
  float v[kPer];
  const int per = D / 32;
  if (a.ids) {
    const int64_t id = a.ids[t];
    const __nv_bfloat16* e = static_cast<const __nv_bfloat16*>(a.embedding) + id * D;
    const __nv_bfloat16* pe =
        a.pos_embedding ? static_cast<const __nv_bfloat16*>(a.pos_embedding) + (int64_t)(a.pos0 + t) * D : nullptr;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      if (j < per) {
        const int i = lane + 32 * j;
        float y = bf(e, i);
        if (pe) y += bf(pe, i);
        v[j] = y;
        xr[i] = y;
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < kPer; ++j)
      if (j < per) v[j] = xr[lane + 32 * j];
  }
  const __nv_bfloat16* w = static_cast<const __nv_bfloat16*>(a.w);
  const __nv_bfloat16* b = static_cast<const __nv_bfloat16*>(a.b);
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out) + (int64_t)t * D;
  float wv[kPer];  // the weights, requested before the reduction
#pragma unroll
  for (int j = 0; j < kPer; ++j) wv[j] = j < per ? bf(w, lane + 32 * j) : 0.f;
  float mean = 0.f, q = 0.f;
  if (a.norm == MIE_NORM_LAYER) {
    float sm = 0.f;
#pragma unroll
    for (int j = 0; j < kPer; ++j)
      if (j < per) sm += v[j];
    mean = warp_sum(sm) / (float)D;
#pragma unroll
    for (int j = 0; j < kPer; ++j)
      if (j < per) q = fmaf(v[j] - mean, v[j] - mean, q);
  } else {
#pragma unroll
    for (int j = 0; j < kPer; ++j)
      if (j < per) q = fmaf(v[j], v[j], q);
  }
  const float rs = rsqrtf(warp_sum(q) / (float)D + a.eps);
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    if (j < per) {
      const int i = lane + 32 * j;
      float y = (v[j] - mean) * rs * wv[j];
      if (b) y += bf(b, i);
      out[i] = __float2bfloat16_rn(y);
    }
  }
}

// One warp per (token, head): hd / 2 RoPE pairs of q and k, hd values of v.
__global__ void __launch_bounds__(kPfThreads) prefill_rope_kv_kernel(const mie_prefill_rope_args a) {
  const int item = blockIdx.x * kPfWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (item >= a.tokens * a.num_heads) return;
  const int t = item / a.num_heads, h = item - t * a.num_heads;
  const int hd = a.head_dim, half = hd / 2, D = a.num_heads * hd;
  const int p = a.pos0 + t;
  const float* row = a.qkv + (int64_t)t * 3 * D;
  const float* qr = row + h * hd;
  const float* kr = row + D + h * hd;
  const float* vr = row + 2 * D + h * hd;
  const int64_t o = ((int64_t)h * a.tokens + t) * hd;  // [H, T, hd]
  __nv_bfloat16* qo = static_cast<__nv_bfloat16*>(a.q_out) + o;
  __nv_bfloat16* ko = static_cast<__nv_bfloat16*>(a.k_out) + o;
  __nv_bfloat16* vo = static_cast<__nv_bfloat16*>(a.v_out) + o;
  int64_t blk = p / a.block_size;
  if (a.block_table) blk = a.block_table[blk];
  const int64_t slot = blk * a.kv_stride_block + (int64_t)h * a.kv_stride_head + (int64_t)(p % a.block_size) * a.kv_stride_tok;
  __nv_bfloat16* kc = static_cast<__nv_bfloat16*>(a.k_cache) + slot;
  __nv_bfloat16* vc = static_cast<__nv_bfloat16*>(a.v_cache) + slot;
  const float* cs = a.rope_cos ? a.rope_cos + (int64_t)p * half : nullptr;
  const float* sn = a.rope_sin ? a.rope_sin + (int64_t)p * half : nullptr;
  for (int j = lane; j < half; j += 32) {
    float q1 = qr[j], q2 = qr[j + half], k1 = kr[j], k2 = kr[j + half];
    if (cs) {
      const float c = cs[j], s = sn[j];
      const float a1 = q1 * c - q2 * s, a2 = q2 * c + q1 * s;
      const float b1 = k1 * c - k2 * s, b2 = k2 * c + k1 * s;
      q1 = a1;
      q2 = a2;
      k1 = b1;
      k2 = b2;
    }
    qo[j] = __float2bfloat16_rn(q1);
    qo[j + half] = __float2bfloat16_rn(q2);
    const __nv_bfloat16 e1 = __float2bfloat16_rn(k1), e2 = __float2bfloat16_rn(k2);
    ko[j] = e1;
    ko[j + half] = e2;
    kc[j] = e1;
    kc[j + half] = e2;
  }
  for (int j = lane; j < hd; j += 32) {
    const __nv_bfloat16 e = __float2bfloat16_rn(vr[j]);
    vo[j] = e;
    vc[j] = e;
  }
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

__global__ void __launch_bounds__(kPfThreads) prefill_route_kernel(const mie_prefill_route_args a) {
  const int t = blockIdx.x * kPfWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (t >= a.tokens) return;
  const int D = a.hidden_dim, E = a.num_experts, per = D / 32;
  const __nv_bfloat16* xr = static_cast<const __nv_bfloat16*>(a.x) + (int64_t)t * D;
  const __nv_bfloat16* rw = static_cast<const __nv_bfloat16*>(a.router_w);
  // the router sees the normalised residual in fp32 (the bf16 copy feeds the
  // expert GEMMs): routing decisions as close to an fp32 forward as possible
  constexpr int kPer = kPfMaxDim / 32;
  float xv[kPer];
  const float* xf = a.x_res + (int64_t)t * D;
#pragma unroll
  for (int j = 0; j < kPer; ++j) xv[j] = j < per ? xf[lane + 32 * j] : 0.f;
  {
    const __nv_bfloat16* nw = static_cast<const __nv_bfloat16*>(a.norm_w);
    const __nv_bfloat16* nb = static_cast<const __nv_bfloat16*>(a.norm_b);
    float mean = 0.f, q = 0.f;
    if (a.norm == MIE_NORM_LAYER) {
      float sm = 0.f;
#pragma unroll
      for (int j = 0; j < kPer; ++j) sm += xv[j];
      mean = warp_sum(sm) / (float)D;
#pragma unroll
      for (int j = 0; j < kPer; ++j)
        if (j < per) q = fmaf(xv[j] - mean, xv[j] - mean, q);
    } else {
#pragma unroll
      for (int j = 0; j < kPer; ++j) q = fmaf(xv[j], xv[j], q);
    }
    const float rs = rsqrtf(warp_sum(q) / (float)D + a.eps);
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      if (j < per) {
        const int i = lane + 32 * j;
        float y = (xv[j] - mean) * rs * bf(nw, i);
        if (nb) y += bf(nb, i);
        xv[j] = y;
      }
    }
  }
  // lane e ends up holding logit e (E <= 32); eight experts at a time, their
  // weight loads and reductions independent of one another
  float mine = -INFINITY;
#pragma unroll 1
  for (int e0 = 0; e0 < E; e0 += 8) {
    float s[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      s[u] = 0.f;
      if (e0 + u < E) {
        const __nv_bfloat16* we = rw + (int64_t)(e0 + u) * D + lane;
#pragma unroll
        for (int j = 0; j < kPer; ++j)
          if (j < per) s[u] = fmaf(xv[j], bf(we, 32 * j), s[u]);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int u = 0; u < 8; ++u) s[u] += __shfl_xor_sync(0xffffffffu, s[u], o);
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (lane == e0 + u) mine = s[u];
  }
  if (a.logits && lane < E) a.logits[(int64_t)t * E + lane] = mine;
  float bv = lane < E ? mine : -INFINITY;
  int bi = lane < E ? lane : 0x7fffffff;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int i0 = bi;
  float cv = (lane < E && lane != i0) ? mine : -INFINITY;
  int ci = (lane < E && lane != i0) ? lane : 0x7fffffff;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, cv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, ci, o);
    if (better(ov, oi, cv, ci)) {
      cv = ov;
      ci = oi;
    }
  }
  const int i1 = ci;
  int r0 = 0, r1 = 0;
  if (lane == 0) {
    const float e1 = expf(cv - bv);
    a.weights[2 * t] = 1.0f / (1.0f + e1);
    a.weights[2 * t + 1] = e1 / (1.0f + e1);
    a.ids_out[2 * t] = i0;
    a.ids_out[2 * t + 1] = i1;
    r0 = i0 * a.group_rows + atomicAdd(a.counts + i0, 1);
    r1 = i1 * a.group_rows + atomicAdd(a.counts + i1, 1);
    a.rows_out[2 * t] = r0;
    a.rows_out[2 * t + 1] = r1;
  }
  r0 = __shfl_sync(0xffffffffu, r0, 0);
  r1 = __shfl_sync(0xffffffffu, r1, 0);
  __nv_bfloat16* g0 = static_cast<__nv_bfloat16*>(a.gathered) + (int64_t)r0 * D;
  __nv_bfloat16* g1 = static_cast<__nv_bfloat16*>(a.gathered) + (int64_t)r1 * D;
  if (((reinterpret_cast<uintptr_t>(xr) | reinterpret_cast<uintptr_t>(g0) | reinterpret_cast<uintptr_t>(g1)) & 15) == 0) {
    // the row in 16-byte pieces (D is a multiple of 32)
    const uint4* src = reinterpret_cast<const uint4*>(xr);
    for (int i = lane; i < D / 8; i += 32) {
      const uint4 v = src[i];
      reinterpret_cast<uint4*>(g0)[i] = v;
      reinterpret_cast<uint4*>(g1)[i] = v;
    }
  } else {
#pragma unroll 4
    for (int j = 0; j < per; ++j) {
      const int i = lane + 32 * j;
      g0[i] = xr[i];
      g1[i] = xr[i];
    }
  }
}

__global__ void __launch_bounds__(kPfThreads) prefill_combine_kernel(const mie_prefill_combine_args a) {
  const int t = blockIdx.x * kPfWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (t >= a.tokens) return;
  const int D = a.hidden_dim;
  const float w0 = a.weights[2 * t], w1 = a.weights[2 * t + 1];
  const float* y0 = a.y + (int64_t)a.rows[2 * t] * a.ldy;
  const float* y1 = a.y + (int64_t)a.rows[2 * t + 1] * a.ldy;
  float4* xr = reinterpret_cast<float4*>(a.x + (int64_t)t * D);
  const float4* a0 = reinterpret_cast<const float4*>(y0);
  const float4* a1 = reinterpret_cast<const float4*>(y1);
#pragma unroll 2
  for (int i = lane; i < D / 4; i += 32) {
    const float4 u = a0[i], v = a1[i];
    float4 x = xr[i];
    x.x = fmaf(w1, v.x, fmaf(w0, u.x, x.x));
    x.y = fmaf(w1, v.y, fmaf(w0, u.y, x.y));
    x.z = fmaf(w1, v.z, fmaf(w0, u.z, x.z));
    x.w = fmaf(w1, v.w, fmaf(w0, u.w, x.w));
    xr[i] = x;
  }
}

unsigned grid_for(int items) { return (unsigned)((items + kPfWarps - 1) / kPfWarps); }

// ---------------------------------------------------------------------------
// Causal attention of the prompt: one CTA per (64-query tile, head), 256
// threads.  Key tiles of 64 up to the diagonal are staged in shared memory as
// fp32 (K transposed, V as rows); thread (ty, tx) holds the scores of queries
// 4 ty .. 4 ty + 3 against keys 4 tx .. 4 tx + 3 and the outputs of those
// queries in dims tx, tx + 16, ...; the online softmax keeps a running max and
// sum per query, reduced over the 16 threads of a query row with shuffles.
// At prompt lengths of hundreds of tokens the whole attention is a few hundred
// MFLOP spread over ~100 CTAs: the kernel is latency bound whatever unit does
// the arithmetic, and plain fp32 FMAs keep the reference's fp32 accumulation.
// ---------------------------------------------------------------------------
constexpr int kAtQ = 64, kAtK = 64, kAtThreads = 256;

template <int HD>
__global__ void __launch_bounds__(kAtThreads) prefill_attention_kernel(const mie_prefill_attn_args a) {
  constexpr int DPT = HD / 16;  // output dims per thread
  extern __shared__ __align__(16) float at_sm[];
  float* qt = at_sm;                 // [HD][kAtQ]   q transposed
  float* kt = qt + HD * kAtQ;        // [HD][kAtK]   k transposed
  float* vs = kt + HD * kAtK;        // [kAtK][HD]
  float* pt = vs + kAtK * HD;        // [kAtK][kAtQ] probabilities transposed
  const int h = blockIdx.y, q0 = blockIdx.x * kAtQ, T = a.tokens, tid = threadIdx.x;
  const int ty = tid >> 4, tx = tid & 15;
  const __nv_bfloat16* qh = static_cast<const __nv_bfloat16*>(a.q) + (int64_t)h * T * HD;
  const __nv_bfloat16* kh = static_cast<const __nv_bfloat16*>(a.k) + (int64_t)h * T * HD;
  const __nv_bfloat16* vh = static_cast<const __nv_bfloat16*>(a.v) + (int64_t)h * T * HD;
  // a tile of 64 rows as 16-byte vectors (8 bf16 of one row each): every
  // thread's loads are issued before any is converted and stored
  constexpr int kVecRow = HD / 8, kVecs = kAtK * kVecRow, kPer = (kVecs + kAtThreads - 1) / kAtThreads;
  auto load_tile = [&](const __nv_bfloat16* base, int r0, uint4* v) {
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int i = tid + u * kAtThreads, r = i / kVecRow, c = i - r * kVecRow;
      v[u] = (i < kVecs && r0 + r < T) ? __ldg(reinterpret_cast<const uint4*>(base + (int64_t)(r0 + r) * HD) + c)
                                       : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  auto unpack = [](uint4 v, float* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      f[2 * e] = __uint_as_float(w[e] << 16);
      f[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
    }
  };
  {
    uint4 qv[kPer];
    load_tile(qh, q0, qv);
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int i = tid + u * kAtThreads, r = i / kVecRow, c = i - r * kVecRow;
      if (i >= kVecs) continue;
      float f[8];
      unpack(qv[u], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) qt[(c * 8 + e) * kAtQ + r] = f[e] * a.scale;
    }
  }
  float m[4], l[4], o[4][DPT];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int j = 0; j < DPT; ++j) o[i][j] = 0.f;
  }
  const int qlast = min(q0 + kAtQ, T) - 1;  // the last query of the tile sees keys up to qlast
  for (int k0 = 0; k0 <= qlast; k0 += kAtK) {
    {
      uint4 kv4[kPer], vv4[kPer];
      load_tile(kh, k0, kv4);  // in flight while the previous tile is finished with
      load_tile(vh, k0, vv4);
      __syncthreads();  // previous tile's k, v, p no longer read (and q staged)
#pragma unroll
      for (int u = 0; u < kPer; ++u) {
        const int i = tid + u * kAtThreads, r = i / kVecRow, c = i - r * kVecRow;
        if (i >= kVecs) continue;
        float f[8], g[8];
        unpack(kv4[u], f);
        unpack(vv4[u], g);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          kt[(c * 8 + e) * kAtK + r] = f[e];
          vs[r * HD + c * 8 + e] = g[e];
        }
      }
    }
    __syncthreads();
    float sc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) sc[i][j] = 0.f;
#pragma unroll 4
    for (int d = 0; d < HD; ++d) {
      const float4 qa = *reinterpret_cast<const float4*>(qt + d * kAtQ + 4 * ty);
      const float4 kb = *reinterpret_cast<const float4*>(kt + d * kAtK + 4 * tx);
      const float qv[4] = {qa.x, qa.y, qa.z, qa.w}, kv[4] = {kb.x, kb.y, kb.z, kb.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) sc[i][j] = fmaf(qv[i], kv[j], sc[i][j]);
    }
    // causal mask and the online softmax of each of this thread's four queries
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qi = q0 + 4 * ty + i;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int kj = k0 + 4 * tx + j;
        if (kj > qi || kj >= T) sc[i][j] = -INFINITY;
        mx = fmaxf(mx, sc[i][j]);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mn = fmaxf(m[i], mx);
      const float alpha = m[i] == -INFINITY ? 0.f : expf(m[i] - mn);
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = mn == -INFINITY ? 0.f : expf(sc[i][j] - mn);
        sc[i][j] = p;
        rs += p;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
      l[i] = l[i] * alpha + rs;
      m[i] = mn;
#pragma unroll
      for (int j = 0; j < DPT; ++j) o[i][j] *= alpha;
#pragma unroll
      for (int j = 0; j < 4; ++j) pt[(4 * tx + j) * kAtQ + 4 * ty + i] = sc[i][j];
    }
    __syncthreads();
    // o += p . v over the tile's keys
#pragma unroll 2
    for (int kj = 0; kj < kAtK; ++kj) {
      const float4 pa = *reinterpret_cast<const float4*>(pt + kj * kAtQ + 4 * ty);
      const float pv[4] = {pa.x, pa.y, pa.z, pa.w};
#pragma unroll
      for (int j = 0; j < DPT; ++j) {
        const float vv = vs[kj * HD + tx + 16 * j];
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i][j] = fmaf(pv[i], vv, o[i][j]);
      }
    }
  }
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int qi = q0 + 4 * ty + i;
    if (qi >= T) continue;
    const float inv = 1.0f / l[i];
#pragma unroll
    for (int j = 0; j < DPT; ++j)
      out[(int64_t)qi * a.ld_out + (int64_t)h * HD + tx + 16 * j] = __float2bfloat16_rn(o[i][j] * inv);
  }
}

// ---------------------------------------------------------------------------
// Causal attention of the prompt on the tensor cores (head_dim 64, bf16): one
// CTA of 128 threads per (128-query tile, head); thread r owns query row r,
// which is TMEM lane r.  For each 64-key tile up to the diagonal:
//   S = Q K^T      tcgen05.mma (M 128, N 64, K 64) into TMEM columns [0, 64);
//   softmax        thread r reads its 64 scores (tcgen05.ld), masks the keys
//                  past its query, updates its running max and sum and writes
//                  its row of P (bf16) to shared memory;
//   O_t = P V      tcgen05.mma (M 128, N 64, K = the tile's 64 keys) into TMEM
//                  columns [64, 128), read back and added to the register O
//                  after the rescale of the running max.
// Operands are K-major tiles in the 128-byte-swizzled layout, written by the
// threads: Q [128 x 64] once, K [64 keys x 64] and V transposed [64 dims x 64
// keys] per tile, double buffered (the next tile's rows are loaded into
// registers while the current tile is reduced).  P is rounded to bf16 for the
// second product, as in flash attention; scores, sums and O stay fp32.
// ---------------------------------------------------------------------------
constexpr int kTcQ = 128, kTcK = 64, kTcThreads = 128, kTcHD = 64;
constexpr uint32_t kTcQBytes = kTcQ * 128u;  // 16 KB: 128 rows of 64 bf16
constexpr uint32_t kTcKBytes = kTcK * 128u;  // 8 KB
constexpr uint32_t kTcVBytes = kTcHD * 128u;  // 8 KB: 64 dims x 64 keys
constexpr uint32_t kTcPBytes = kTcQ * 128u;  // 16 KB
constexpr uint32_t kTcSmem = kTcQBytes + 2 * kTcKBytes + 2 * kTcVBytes + kTcPBytes + 1024u;  // + alignment
constexpr uint32_t kTcCols = 128;  // TMEM: S [0, 64), O_t [64, 128)

// Byte offset of 16-byte chunk c of row r in a K-major 128-byte-swizzled tile
// (rows of 128 bytes; chunk c of row r sits at chunk c ^ (r mod 8)).
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return (uint32_t)r * 128u + ((uint32_t)(c ^ (r & 7)) << 4);
}

__global__ void __launch_bounds__(kTcThreads, 1) prefill_attention_tc_kernel(const mie_prefill_attn_args a) {
  extern __shared__ uint8_t tc_raw[];
  uint8_t* sq = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* skv = sq + kTcQBytes;  // [2][K | V^T]
  uint8_t* sp = skv + 2 * (kTcKBytes + kTcVBytes);
  __shared__ __align__(8) uint64_t bar_s, bar_o;
  __shared__ uint32_t tmem_s;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int h = blockIdx.y, q0 = blockIdx.x * kTcQ, T = a.tokens;
  const __nv_bfloat16* qh = static_cast<const __nv_bfloat16*>(a.q) + (int64_t)h * T * kTcHD;
  const __nv_bfloat16* kh = static_cast<const __nv_bfloat16*>(a.k) + (int64_t)h * T * kTcHD;
  const __nv_bfloat16* vh = static_cast<const __nv_bfloat16*>(a.v) + (int64_t)h * T * kTcHD;
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  if (tid == 0) {
    mbar_init(&bar_s, 1u);
    mbar_init(&bar_o, 1u);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(&tmem_s, kTcCols);
  // Q tile (rows past T are zero)
#pragma unroll
  for (int u = 0; u < kTcQ * 8 / kTcThreads; ++u) {
    const int i = tid + u * kTcThreads, r = i >> 3, c = i & 7;
    const uint4 v = q0 + r < T ? __ldg(reinterpret_cast<const uint4*>(qh + (int64_t)(q0 + r) * kTcHD) + c) : zero;
    *reinterpret_cast<uint4*>(sq + sw128_off(r, c)) = v;
  }
  // K rows: chunk (key i >> 3, piece i & 7), four per thread; V rows: thread
  // t holds dims [32 (t >> 6), + 32) of key t & 63 (the transposed store of a
  // warp then writes 32 consecutive keys of one row: no bank conflict)
  uint4 kr[4], vr[4];
  const int vkey = tid & 63, vd0 = (tid >> 6) * 32;
  auto load_kv = [&](int k0) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = tid + u * kTcThreads, r = i >> 3, c = i & 7;
      kr[u] = k0 + r < T ? __ldg(reinterpret_cast<const uint4*>(kh + (int64_t)(k0 + r) * kTcHD) + c) : zero;
      vr[u] = k0 + vkey < T
                  ? __ldg(reinterpret_cast<const uint4*>(vh + (int64_t)(k0 + vkey) * kTcHD + vd0) + u)
                  : zero;
    }
  };
  auto store_kv = [&](int buf) {
    uint8_t* sk = skv + (uint32_t)buf * (kTcKBytes + kTcVBytes);
    uint8_t* sv = sk + kTcKBytes;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = tid + u * kTcThreads, r = i >> 3, c = i & 7;
      *reinterpret_cast<uint4*>(sk + sw128_off(r, c)) = kr[u];
      const uint32_t w[4] = {vr[u].x, vr[u].y, vr[u].z, vr[u].w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int d = vd0 + 8 * u + e;  // row of V^T
        const uint16_t bits = (uint16_t)(e & 1 ? w[e >> 1] >> 16 : w[e >> 1] & 0xffffu);
        *reinterpret_cast<uint16_t*>(sv + sw128_off(d, vkey >> 3) + (vkey & 7) * 2) = bits;
      }
    }
  };
  const int qi = q0 + tid;  // this thread's query
  const int klast = min(q0 + kTcQ, T) - 1;  // the tile's last query sees keys up to klast
  const int nkt = klast / kTcK + 1;
  load_kv(0);
  store_kv(0);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_s;
  const uint32_t tlane = tmem + ((uint32_t)(warp * 32) << 16);
  constexpr uint32_t idesc = idesc_bf16(kTcK, kTcQ);  // both products: M 128, N 64
  const float scale = a.scale;
  float o[kTcHD], m = -INFINITY, l = 0.f;
#pragma unroll
  for (int d = 0; d < kTcHD; ++d) o[d] = 0.f;
  // `ok` (every wait succeeded) is made CTA-uniform at each block barrier, so
  // every thread leaves the loop at the same barrier
  bool ok = true;
#pragma unroll 1
  for (int j = 0; j < nkt; ++j) {
    const int k0 = j * kTcK, buf = j & 1;
    const uint8_t* sk = skv + (uint32_t)buf * (kTcKBytes + kTcVBytes);
    const uint8_t* sv = sk + kTcKBytes;
    // the tile's K / V^T (and Q) stores by every thread, then the MMAs
    fence_proxy_async_smem();
    tc_fence_before();
    ok = __syncthreads_and(ok) != 0;
    tc_fence_after();
    if (!ok) break;
    if (tid == 0) {
#pragma unroll
      for (int kk = 0; kk < kTcHD / 16; ++kk)
        tc_mma(tmem, sw128_desc(sq, 32u * kk), sw128_desc(sk, 32u * kk), idesc, kk ? 1u : 0u);
      tc_commit(&bar_s);
    }
    if (j + 1 < nkt) load_kv(k0 + kTcK);  // the next tile's rows in flight during this one
    ok = mbar_wait(&bar_s, (uint32_t)(j & 1), a.status);
    tc_fence_after();
    float s[kTcK];
    tmem_ld32(tlane, s);
    tmem_ld32(tlane + 32, s + 32);
    // causal mask, online softmax of this thread's row, P row (bf16) to shared memory
    float mx = -INFINITY;
#pragma unroll
    for (int c = 0; c < kTcK; ++c) {
      s[c] = (k0 + c <= qi && k0 + c < T) ? s[c] * scale : -INFINITY;
      mx = fmaxf(mx, s[c]);
    }
    const float mn = fmaxf(m, mx);
    const float alpha = m == -INFINITY ? 0.f : expf(m - mn);
    float rs = 0.f;
#pragma unroll
    for (int c = 0; c < kTcK; c += 8) {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const float p0 = mn == -INFINITY ? 0.f : expf(s[c + e] - mn);
        const float p1 = mn == -INFINITY ? 0.f : expf(s[c + e + 1] - mn);
        rs += p0 + p1;
        const __nv_bfloat162 pb = __floats2bfloat162_rn(p0, p1);
        w[e >> 1] = *reinterpret_cast<const uint32_t*>(&pb);
      }
      *reinterpret_cast<uint4*>(sp + sw128_off(tid, c >> 3)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    l = fmaf(l, alpha, rs);
    m = mn;
    if (j + 1 < nkt) store_kv(buf ^ 1);  // the other buffer: its MMAs completed last iteration
    fence_proxy_async_smem();
    tc_fence_before();
    ok = __syncthreads_and(ok) != 0;
    tc_fence_after();
    if (!ok) break;
    if (tid == 0) {
#pragma unroll
      for (int kk = 0; kk < kTcK / 16; ++kk)
        tc_mma(tmem + kTcK, sw128_desc(sp, 32u * kk), sw128_desc(sv, 32u * kk), idesc, kk ? 1u : 0u);
      tc_commit(&bar_o);
    }
    ok = mbar_wait(&bar_o, (uint32_t)(j & 1), a.status);
    tc_fence_after();
    float pv[kTcHD];
    tmem_ld32(tlane + kTcK, pv);
    tmem_ld32(tlane + kTcK + 32, pv + 32);
#pragma unroll
    for (int d = 0; d < kTcHD; ++d) o[d] = fmaf(o[d], alpha, pv[d]);
  }
  if (ok && qi < T) {
    const float inv = 1.0f / l;
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out) + (int64_t)qi * a.ld_out + (int64_t)h * kTcHD;
#pragma unroll
    for (int d = 0; d < kTcHD; d += 8) {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const __nv_bfloat162 ob = __floats2bfloat162_rn(o[d + e] * inv, o[d + e + 1] * inv);
        w[e >> 1] = *reinterpret_cast<const uint32_t*>(&ob);
      }
      *reinterpret_cast<uint4*>(out + d) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_free(tmem, kTcCols);
  }
}

int prefill_attention_tc_launch(const mie_prefill_attn_args& a, cudaStream_t st) {
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(prefill_attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem);
    attr = true;
  }
  return launch(prefill_attention_tc_kernel, dim3((unsigned)((a.tokens + kTcQ - 1) / kTcQ), (unsigned)a.num_heads),
                dim3(kTcThreads), kTcSmem, st, false, a);
}

template <int HD>
int prefill_attention_launch(const mie_prefill_attn_args& a, cudaStream_t st) {
  const uint32_t smem = (uint32_t)sizeof(float) * (2 * HD * kAtQ + kAtK * HD + kAtK * kAtQ);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(prefill_attention_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr = true;
  }
  return launch(prefill_attention_kernel<HD>, dim3((unsigned)((a.tokens + kAtQ - 1) / kAtQ), (unsigned)a.num_heads),
                dim3(kAtThreads), smem, st, false, a);
}

}  // namespace

int prefill_attention(const mie_prefill_attn_args& a, cudaStream_t st) {
  if (a.tokens <= 0 || a.num_heads <= 0 || !a.q || !a.k || !a.v || !a.out || a.ld_out < (int64_t)a.num_heads * a.head_dim)
    return MIE_ERR_INVALID;
  // head_dim 64 with 16-byte aligned rows: the tensor-core kernel
  const bool rows16 = ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) |
                        reinterpret_cast<uintptr_t>(a.v) | reinterpret_cast<uintptr_t>(a.out)) % 16 == 0) &&
                      a.ld_out % 8 == 0;
  if (a.head_dim == kTcHD && rows16) return prefill_attention_tc_launch(a, st);
  switch (a.head_dim) {
    case 64: return prefill_attention_launch<64>(a, st);
    case 96: return prefill_attention_launch<96>(a, st);
    case 128: return prefill_attention_launch<128>(a, st);
    default: return MIE_ERR_UNSUPPORTED;
  }
}

int prefill_norm(const mie_prefill_norm_args& a, cudaStream_t st) {
  if (a.tokens <= 0 || a.hidden_dim <= 0 || a.hidden_dim % 32 || a.hidden_dim > kPfMaxDim || !a.x || !a.w ||
      !a.out || (a.ids && !a.embedding))
    return MIE_ERR_INVALID;
  return launch(prefill_norm_kernel, dim3(grid_for(a.tokens)), dim3(kPfThreads), 0, st, false, a);
}

int prefill_rope_kv(const mie_prefill_rope_args& a, cudaStream_t st) {
  if (a.tokens <= 0 || a.num_heads <= 0 || a.head_dim <= 0 || a.head_dim % 2 || !a.qkv || !a.q_out || !a.k_out ||
      !a.v_out || !a.k_cache || !a.v_cache || a.block_size <= 0 || (a.rope_cos && !a.rope_sin))
    return MIE_ERR_INVALID;
  return launch(prefill_rope_kv_kernel, dim3(grid_for(a.tokens * a.num_heads)), dim3(kPfThreads), 0, st, false, a);
}

int prefill_route(const mie_prefill_route_args& a, cudaStream_t st) {
  if (a.tokens <= 0 || a.hidden_dim % 32 || a.hidden_dim > kPfMaxDim || a.num_experts < 2 || a.num_experts > 32 ||
      a.group_rows < a.tokens || !a.x || !a.x_res || !a.norm_w || !a.router_w || !a.counts || !a.weights ||
      !a.ids_out || !a.rows_out || !a.gathered)
    return MIE_ERR_INVALID;
  return launch(prefill_route_kernel, dim3(grid_for(a.tokens)), dim3(kPfThreads), 0, st, false, a);
}

int prefill_combine(const mie_prefill_combine_args& a, cudaStream_t st) {
  if (a.tokens <= 0 || a.hidden_dim <= 0 || a.hidden_dim % 4 || a.ldy % 4 || !a.x || !a.y || !a.weights || !a.rows ||
      a.ldy < a.hidden_dim || (reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.y)) % 16)
    return MIE_ERR_INVALID;
  return launch(prefill_combine_kernel, dim3(grid_for(a.tokens)), dim3(kPfThreads), 0, st, false, a);
}

}  // namespace mie
