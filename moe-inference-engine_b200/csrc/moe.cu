// Fused top-2 MoE decode layer for one token (batch one), sm_100a.
//
// Replaces the reference's three Triton launches (router + top-2, selected
// W1 + activation, selected W2 + weighted combine; src/moe_engine/fused_moe.py
// :120-262) with ONE persistent launch:
//
//   prologue (every CTA, redundantly): x -> norm -> router GEMV (8 x D) ->
//       top-2 by repeated argmax (ties -> lower id) -> 2-way softmax.
//   up phase: the 2 x Hx hidden units of the two selected experts are split
//       evenly over the grid; each CTA streams only its rows of W1 (and W3 for
//       SwiGLU) with TMA bulk copies and writes h = act(W1 x + b1) (* W3 x).
//   grid barrier (bounded; the down-phase weights were prefetched before it).
//   down phase: the D output rows are split over the grid; each CTA streams
//       its rows of both selected experts' W2 and writes
//       out = (x) + sum_r w_r (W2[e_r] h_r + b2[e_r]).
//
// Only the selected experts' bytes are read: router + 2 x (W1 [, W3], W2).
// The reduction order is fixed, so results are bit-reproducible.
#include "kernels.h"
#include "stream.cuh"

namespace mie {

namespace {

enum : uint8_t { kTagUpA = 0, kTagUpB = 1, kTagDown = 2 };
constexpr int kMaxChunks = 96;

__device__ __forceinline__ float gelu_erf(float v) { return 0.5f * v * (1.0f + erff(v * 0.7071067811865476f)); }
__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }

template <typename W>
__global__ void __launch_bounds__(256) moe_decode_kernel(const mie_moe_args a, MoeLayout L) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int D = a.hidden_dim, Hx = a.expert_hidden_dim, E = a.num_experts;
  const int G = gridDim.x, c = blockIdx.x, tid = threadIdx.x;
  const bool swiglu = a.act == MIE_ACT_SWIGLU;

  Ring R;
  R.bar = reinterpret_cast<uint64_t*>(smem + L.off_bar);
  R.data = smem + L.off_ring;
  R.nslot = L.nslot;
  R.slot_bytes = L.slot_bytes;
  uint64_t* router_bar = reinterpret_cast<uint64_t*>(smem + L.off_bar) + L.nslot;
  W* router_s = reinterpret_cast<W*>(smem + L.off_router);
  float* xs = reinterpret_cast<float*>(smem + L.off_x);
  float* hs = reinterpret_cast<float*>(smem + L.off_h);       // [2, Hx]
  float* resA = reinterpret_cast<float*>(smem + L.off_res);   // up results (gate / fc1)
  float* resB = resA + L.max_units;                           // up results (up)
  float* resD = resB + L.max_units;                           // down results [2][max_rows]
  Chunk* chunks = reinterpret_cast<Chunk*>(smem + L.off_chunks);
  __shared__ float red[8];
  __shared__ float logits_s[32];
  __shared__ int ids_s[2];
  __shared__ float wts_s[2];
  __shared__ int nchunk_s, first_down_s, issued_s;

  const uint64_t pol = policy_evict_first();
  const uint32_t router_bytes = (uint32_t)(E * D * sizeof(W));
  if (tid == 0) {
    ring_init(R);
    mbar_init(router_bar, 1);
    fence_barrier_init();
    // Router weights are static: fetch them before waiting on the producer grid.
    mbar_arrive_expect_tx(router_bar, router_bytes);
    for (uint32_t off = 0; off < router_bytes; off += kBulkMax)
      bulk_g2s(reinterpret_cast<uint8_t*>(router_s) + off, static_cast<const uint8_t*>(a.router_w) + off,
               min(kBulkMax, router_bytes - off), router_bar);
  }
  __syncthreads();

  pdl_wait();
  if (skip_requested(a.skip)) {
    if (tid == 0) mbar_wait(router_bar, 0, a.status);
    __syncthreads();
    pdl_trigger();
    return;
  }

  // ---- prologue: norm + router + top-2 (identical in every CTA) ----
  load_and_norm(xs, a.x, a.x_dtype, nullptr, D, a.norm, a.eps, a.norm_w, a.norm_b, a.dtype, red);
  const bool rok = mbar_wait(router_bar, 0, a.status);
  if (!__syncthreads_and(rok)) return;
  {
    const int lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    constexpr int PV = Elem<W>::kPerVec;
    const int nvec = D / PV;
    for (int e = warp; e < E; e += nw) {
      const uint4* row = reinterpret_cast<const uint4*>(router_s) + (size_t)e * nvec;
      float acc = 0.f;
      for (int v = lane; v < nvec; v += kWarp) acc = dot_vec(row[v], xs + v * PV, acc, (const W*)nullptr);
      acc = warp_sum(acc);
      if (lane == 0) logits_s[e] = acc;
    }
  }
  __syncthreads();
  if (tid == 0) {
    // Repeated argmax: strict '>' while scanning ascending ids keeps the lower
    // id on ties (fused_moe.py:146-150).
    int i0 = 0;
    for (int e = 1; e < E; ++e)
      if (logits_s[e] > logits_s[i0]) i0 = e;
    int i1 = (i0 == 0) ? 1 : 0;
    for (int e = 0; e < E; ++e)
      if (e != i0 && logits_s[e] > logits_s[i1]) i1 = e;
    const float l0 = logits_s[i0], l1 = logits_s[i1];
    const float e1 = expf(l1 - l0);  // l0 >= l1: stable 2-way softmax
    const float den = 1.0f + e1;
    ids_s[0] = i0;
    ids_s[1] = i1;
    wts_s[0] = 1.0f / den;
    wts_s[1] = e1 / den;
    if (c == 0) {
      if (a.router_logits)
        for (int e = 0; e < E; ++e) a.router_logits[e] = logits_s[e];
      if (a.expert_ids) {
        a.expert_ids[0] = i0;
        a.expert_ids[1] = i1;
      }
      if (a.route_weights) {
        a.route_weights[0] = wts_s[0];
        a.route_weights[1] = wts_s[1];
      }
    }
  }
  __syncthreads();
  if (L.route_only) {
    pdl_trigger();
    return;
  }

  // ---- chunk list: up rows of both selected experts, then down rows ----
  const int ebase = a.expert_base;
  const int ecount = a.expert_count > 0 ? a.expert_count : E;
  const uint32_t row_up = (uint32_t)(D * sizeof(W));
  const uint32_t row_dn = (uint32_t)(Hx * sizeof(W));
  const int cap_up = (int)(R.slot_bytes / row_up);
  const int cap_dn = (int)(R.slot_bytes / row_dn);
  int u0, u1, r0, r1;
  split_range(2 * Hx, c, G, &u0, &u1);
  split_range(D, c, G, &r0, &r1);
  bool local[2];
  int le[2];
  for (int r = 0; r < 2; ++r) {
    le[r] = ids_s[r] - ebase;
    local[r] = le[r] >= 0 && le[r] < ecount;
  }
  if (tid == 0) {
    int n = 0;
    bool ok = true;
    for (int r = 0; r < 2; ++r) {
      // units of slot r inside [u0, u1)
      const int lo = max(u0, r * Hx), hi = min(u1, (r + 1) * Hx);
      if (lo >= hi || !local[r]) continue;
      const int64_t erow = (int64_t)le[r] * Hx;
      ok &= push_rows(chunks, &n, kMaxChunks, a.w1, erow + (lo - r * Hx), hi - lo, row_up, cap_up, kTagUpA,
                      (uint8_t)r, lo - u0);
      if (swiglu)
        ok &= push_rows(chunks, &n, kMaxChunks, a.w3, erow + (lo - r * Hx), hi - lo, row_up, cap_up, kTagUpB,
                        (uint8_t)r, lo - u0);
    }
    first_down_s = n;
    for (int r = 0; r < 2; ++r) {
      if (r1 <= r0 || !local[r]) continue;
      ok &= push_rows(chunks, &n, kMaxChunks, a.w2, (int64_t)le[r] * D + r0, r1 - r0, row_dn, cap_dn, kTagDown,
                      (uint8_t)r, 0);
    }
    if (!ok) {
      set_status(a.status, MIE_ERR_INVALID);
      n = 0;
      first_down_s = 0;
    }
    nchunk_s = n;
    const int first = min(n, R.nslot);
    for (int i = 0; i < first; ++i) ring_issue(R, chunks[i], i, pol);
    issued_s = first;
  }
  for (int i = tid; i < 2 * L.max_rows; i += blockDim.x) resD[i] = 0.f;
  __syncthreads();
  const int n = nchunk_s, first_down = first_down_s;

  bool synced = false;
  auto finish_up_and_sync = [&]() {
    // h for this CTA's units -> global scratch, then the grid barrier.
    for (int k = tid; k < u1 - u0; k += blockDim.x) {
      const int u = u0 + k, r = u / Hx, j = u - r * Hx;
      if (!local[r]) continue;
      float pre = resA[k];
      if (a.b1) pre += load_any(a.b1, a.dtype, (int64_t)le[r] * Hx + j);
      const float h = swiglu ? silu(pre) * resB[k] : gelu_erf(pre);
      a.hidden[(int64_t)r * Hx + j] = h;
    }
    const bool ok = grid_barrier(a.sync, (uint32_t)G, a.status);
    synced = true;
    pdl_trigger();
    if (ok)
      for (int i = tid; i < 2 * Hx; i += blockDim.x) hs[i] = __ldcg(a.hidden + i);
    __syncthreads();
  };

  const bool ok = ring_consume(R, chunks, n, issued_s, pol, a.status, [&](int i, const Chunk& ch, const uint8_t* s) {
    if (i == first_down && !synced) finish_up_and_sync();
    if (ch.tag == kTagDown) {
      float* dst = resD + ch.sub * L.max_rows;
      chunk_dot_rows<W>(s, ch.rows, Hx, hs + ch.sub * Hx, [&](int row, float v) { dst[ch.out + row] = v; });
    } else {
      float* dst = (ch.tag == kTagUpA ? resA : resB);
      chunk_dot_rows<W>(s, ch.rows, D, xs, [&](int row, float v) { dst[ch.out + row] = v; });
    }
  });
  if (!synced) finish_up_and_sync();
  if (!ok) return;

  // ---- epilogue: weighted combine (+ residual) for rows [r0, r1) ----
  for (int k = tid; k < r1 - r0; k += blockDim.x) {
    const int row = r0 + k;
    float y = 0.f;
    for (int r = 0; r < 2; ++r) {
      if (!local[r]) continue;
      float v = resD[r * L.max_rows + k];
      if (a.b2) v += load_any(a.b2, a.dtype, (int64_t)le[r] * D + row);
      y = fmaf(wts_s[r], v, y);
    }
    if (a.residual) y += load_any(a.x, a.x_dtype, row);
    store_any(a.out, a.out_dtype, row, y);
  }
}

}  // namespace

MoeLayout moe_layout(const mie_moe_args& a, int grid, int slot_bytes, int nslot) {
  const int wsz = a.dtype == MIE_BF16 ? 2 : 4;
  MoeLayout L{};
  L.nslot = nslot;
  L.slot_bytes = (uint32_t)slot_bytes;
  L.max_units = (2 * a.expert_hidden_dim + grid - 1) / grid + 1;
  L.max_rows = (a.hidden_dim + grid - 1) / grid + 1;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    off = (off + 127) & ~size_t(127);
    const size_t at = off;
    off += bytes;
    return (uint32_t)at;
  };
  L.off_bar = take(sizeof(uint64_t) * (nslot + 1));
  L.off_ring = take((size_t)nslot * slot_bytes);
  L.off_router = take((size_t)a.num_experts * a.hidden_dim * wsz);
  L.off_x = take(sizeof(float) * a.hidden_dim);
  L.off_h = take(sizeof(float) * 2 * a.expert_hidden_dim);
  L.off_res = take(sizeof(float) * (2 * L.max_units + 2 * L.max_rows));
  L.off_chunks = take(sizeof(Chunk) * kMaxChunks);
  L.smem = (uint32_t)((off + 127) & ~size_t(127));
  return L;
}

int moe_decode_launch(const mie_moe_args& a, const MoeLayout& L, int grid, cudaStream_t st, bool pdl) {
  void (*k)(const mie_moe_args, MoeLayout) =
      a.dtype == MIE_BF16 ? moe_decode_kernel<__nv_bfloat16> : moe_decode_kernel<float>;
  return launch(k, dim3(grid), dim3(256), L.smem, st, pdl, a, L);
}

void moe_set_attributes() {
  set_max_smem(moe_decode_kernel<__nv_bfloat16>);
  set_max_smem(moe_decode_kernel<float>);
}

}  // namespace mie
