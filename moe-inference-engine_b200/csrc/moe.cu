// Fused top-2 MoE decode layer for one token (batch one), sm_100a.
//
// Replaces the reference's three Triton launches (router + top-2, selected
// W1 + activation, selected W2 + weighted combine; src/moe_engine/fused_moe.py
// :120-262) with ONE persistent launch:
//
//   prologue (every CTA, redundantly): x -> norm -> router GEMV (E x D) ->
//       top-2 by repeated argmax (ties -> lower id) -> 2-way softmax.  The
//       router rows are loaded into registers before the PDL wait.
//   right after routing every warp requests its up rows (W1 [, W3]) of the two
//       selected experts AND its down rows (W2), all at once, into registers.
//   up phase: the 2 x Hx hidden units are split evenly over the grid; a warp
//       reduces its unit's rows and writes h = act(W1 x + b1) (* W3 x).
//   grid barrier (monotonic counter).
//   down phase: the D output rows (x 2 experts) are split over the grid; a
//       warp dots its (already loaded) W2 row with h; the CTA combines
//       out = (x) + sum_r w_r (W2[e_r] h_r + b2[e_r]).
//
// Only the selected experts' bytes are read: router + 2 x (W1 [, W3], W2).
// Every reduction has a fixed order, so results are bit-reproducible.
#include "kernels.h"
#include "stream.cuh"

namespace mie {

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ float gelu_erf(float v) { return 0.5f * v * (1.0f + erff(v * 0.7071067811865476f)); }
__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }

__device__ __forceinline__ const uint4* row_ptr(const void* base, int64_t row, int64_t row_bytes) {
  return reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(base) + row * row_bytes);
}

template <typename W>
__global__ void __launch_bounds__(kThreads) moe_decode_kernel(const mie_moe_args a, MoeLayout L) {
  extern __shared__ __align__(16) float smem_f[];
  constexpr int PV = Elem<W>::kPerVec;
  const int D = a.hidden_dim, Hx = a.expert_hidden_dim, E = a.num_experts;
  const int G = gridDim.x, c = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool swiglu = a.act == MIE_ACT_SWIGLU;
  float* xs = smem_f;                 // [D] normalised input
  float* hs = xs + L.off_h;           // [2, Hx] expert activations
  float* resD = xs + L.off_res;       // [2, max_rows] down-projection results
  __shared__ float red[kWarps];
  __shared__ float logits_s[32];
  __shared__ int ids_s[2];
  __shared__ float wts_s[2];
  __shared__ uint64_t target_s;

  uint64_t* ctr = reinterpret_cast<uint64_t*>(a.sync);
  const int nvec_d = D / PV, nvec_h = Hx / PV;  // vectors per up row / per down row
  const int64_t rb_d = (int64_t)D * sizeof(W), rb_h = (int64_t)Hx * sizeof(W);
  const bool up_regs = nvec_d <= Seg<W>::kVecs;  // one segment: keep rows in registers
  const bool dn_regs = nvec_h <= Seg<W>::kVecs;

  // Router rows are static: request them before waiting on the producer grid.
  RowRegs<W> rr[2];
  if (up_regs) {
    for (int k = 0; k < 2; ++k)
      if (warp + kWarps * k < E) row_load<W>(rr[k], row_ptr(a.router_w, warp + kWarps * k, rb_d), nvec_d, 0);
  }
  if (tid == 0 && !L.route_only) target_s = grid_sync_target(ctr, (uint32_t)G);

  pdl_wait();
  if (skip_requested(a.skip)) {
    pdl_trigger();
    return;
  }
  // expert parallel with the all-reduce fused in: this launch's call number
  __shared__ uint32_t ptag_s;
  const bool peer = a.peer_world > 1 && !L.route_only;
  if (peer && tid == 0) ptag_s = peer_tag(a);

  // ---- prologue: norm + router + top-2 (identical in every CTA) ----
  load_and_norm(xs, a.x, a.x_dtype, nullptr, D, a.norm, a.eps, a.norm_w, a.norm_b, a.dtype, red);
  float xr[Seg<W>::kNV * PV];
  if (up_regs) load_x_regs<W>(xr, xs, nvec_d);
  for (int k = 0; k < 2; ++k) {
    const int e = warp + kWarps * k;
    if (e < E) {
      const float v = up_regs ? warp_sum(row_dot_regs<W>(rr[k], xr))
                              : warp_row_dot<W>(row_ptr(a.router_w, e, rb_d), nvec_d, xs);
      if (lane == 0) logits_s[e] = v;
    }
  }
  __syncthreads();
  if (tid == 0) {
    int i0, i1;
    top2_route(logits_s, E, &i0, &i1, &wts_s[0], &wts_s[1]);
    ids_s[0] = i0;
    ids_s[1] = i1;
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

  // ---- this CTA's work: up units [u0, u1), down rows [r0, r1) x 2 experts ----
  const int ebase = a.expert_base;
  const int ecount = a.expert_count > 0 ? a.expert_count : E;
  int u0, u1, r0, r1;
  split_range(2 * Hx, c, G, &u0, &u1);
  split_range(D, c, G, &r0, &r1);
  const int nu = u1 - u0, nr = r1 - r0;
  int le[2];
  bool local[2];
  for (int r = 0; r < 2; ++r) {
    le[r] = ids_s[r] - ebase;
    local[r] = le[r] >= 0 && le[r] < ecount;
  }
  // unit k (of this CTA) -> slot r, hidden index j
  auto unit = [&](int k, int* r, int* j) {
    const int u = u0 + k;
    *r = u / Hx;
    *j = u - *r * Hx;
  };
  // down pair p -> slot r = p / nr, output row r0 + p % nr
  auto pair_slot = [&](int p) { return p / nr; };

  // Request the first up unit and the first down pair of this warp together.
  RowRegs<W> wg, wu, wd;
  int r_first, j_first;
  const bool up0 = warp < nu;
  if (up0) unit(warp, &r_first, &j_first);
  const bool up0_ok = up0 && local[r_first];
  if (up_regs && up0_ok) {
    const int64_t row = (int64_t)le[r_first] * Hx + j_first;
    row_load<W>(wg, row_ptr(a.w1, row, rb_d), nvec_d, 0);
    if (swiglu) row_load<W>(wu, row_ptr(a.w3, row, rb_d), nvec_d, 0);
  }
  const int np = 2 * nr;
  const bool dn0 = warp < np && local[pair_slot(warp)];
  if (dn_regs && dn0) {
    const int r = pair_slot(warp);
    row_load<W>(wd, row_ptr(a.w2, (int64_t)le[r] * D + r0 + warp % nr, rb_h), nvec_h, 0);
  }

  // ---- up phase ----
  for (int k = warp; k < nu; k += kWarps) {
    int r, j;
    unit(k, &r, &j);
    if (!local[r]) continue;
    const int64_t row = (int64_t)le[r] * Hx + j;
    float g, u = 0.f;
    if (up_regs) {
      if (k != warp) {
        row_load<W>(wg, row_ptr(a.w1, row, rb_d), nvec_d, 0);
        if (swiglu) row_load<W>(wu, row_ptr(a.w3, row, rb_d), nvec_d, 0);
      }
      g = warp_sum(row_dot_regs<W>(wg, xr));
      if (swiglu) u = warp_sum(row_dot_regs<W>(wu, xr));
    } else {
      g = warp_row_dot<W>(row_ptr(a.w1, row, rb_d), nvec_d, xs);
      if (swiglu) u = warp_row_dot<W>(row_ptr(a.w3, row, rb_d), nvec_d, xs);
    }
    if (lane == 0) {
      if (a.b1) g += load_any(a.b1, a.dtype, row);
      a.hidden[(int64_t)r * Hx + j] = swiglu ? silu(g) * u : gelu_erf(g);
    }
  }

  // ---- grid barrier: every CTA's h is in global memory ----
  const bool ok = grid_sync(ctr, target_s, a.status);
  pdl_trigger();
  if (!ok) return;
  for (int i = tid; i < 2 * Hx; i += blockDim.x) hs[i] = __ldcg(a.hidden + i);
  __syncthreads();

  // ---- down phase ----
  for (int p = warp; p < np; p += kWarps) {
    const int r = pair_slot(p), row = r0 + p % nr;
    if (!local[r]) continue;
    float v;
    if (dn_regs) {
      if (p != warp) row_load<W>(wd, row_ptr(a.w2, (int64_t)le[r] * D + row, rb_h), nvec_h, 0);
      v = warp_sum(row_dot<W>(wd, hs + (size_t)r * Hx, nvec_h, 0));
    } else {
      v = warp_row_dot<W>(row_ptr(a.w2, (int64_t)le[r] * D + row, rb_h), nvec_h, hs + (size_t)r * Hx);
    }
    if (lane == 0) resD[p] = v;
  }
  __syncthreads();

  // ---- epilogue: weighted combine (+ residual) for rows [r0, r1) ----
  for (int k = tid; k < nr; k += blockDim.x) {
    const int row = r0 + k;
    float y = 0.f;
    for (int r = 0; r < 2; ++r) {
      if (!local[r]) continue;
      float v = resD[r * nr + k];
      if (a.b2) v += load_any(a.b2, a.dtype, (int64_t)le[r] * D + row);
      y = fmaf(wts_s[r], v, y);
    }
    if (peer) y = peer_row_sum(a, D, row, y, ptag_s);  // every rank's partial of this row
    if (a.residual) y += load_any(a.x, a.x_dtype, row);
    store_any(a.out, a.out_dtype, row, y);
  }
  // every CTA read the counter before the grid barrier
  if (peer && c == 0 && tid == 0) *reinterpret_cast<volatile uint32_t*>(a.peer_seq) = ptag_s;
}

}  // namespace

MoeLayout moe_layout(const mie_moe_args& a, int grid, int, int) {
  MoeLayout L{};
  L.max_rows = (a.hidden_dim + grid - 1) / grid + 1;
  const uint32_t d4 = (uint32_t)((a.hidden_dim + 3) & ~3);
  const uint32_t h4 = (uint32_t)((2 * a.expert_hidden_dim + 3) & ~3);
  L.off_h = d4;                 // offsets in floats
  L.off_res = d4 + h4;
  L.smem = (L.off_res + 2 * (uint32_t)L.max_rows) * (uint32_t)sizeof(float);
  return L;
}

int moe_decode_launch(const mie_moe_args& a, const MoeLayout& L, int grid, cudaStream_t st, bool pdl) {
  void (*k)(const mie_moe_args, MoeLayout) =
      a.dtype == MIE_BF16 ? moe_decode_kernel<__nv_bfloat16> : moe_decode_kernel<float>;
  return launch(k, dim3(grid), dim3(kThreads), L.smem, st, pdl, a, L);
}

void moe_set_attributes() {
  set_max_smem(moe_decode_kernel<__nv_bfloat16>);
  set_max_smem(moe_decode_kernel<float>);
}

}  // namespace mie
