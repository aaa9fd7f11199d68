// Fused top-2 MoE decode layer with groupwise-quantized expert weights
// (int8, or int4 two per byte), batch one, sm_100a.
//
// The reference has no quantized path: its roadmap lists "Int8 and int4
// groupwise expert weights" (moe-inference-engine.md:36) without code.  This
// layer computes what src/moe_engine/fused_moe.py:312-380 computes -- router
// GEMV, top-2 with ties to the lower id, 2-way softmax, the selected experts,
// weighted combine -- with every expert weight w[r][i] replaced by
// scale[r][i / group] * q[r][i]: symmetric absmax groups along the reduction
// dimension of each row, q in [-127, 127] (int8) or [-7, 7] (int4, the even
// element in the low nibble of each byte).  Only the selected experts' bytes
// are read: int8 halves and int4 quarters the bytes of the bf16 layer.
//
// Structure as the bf16 kernel (moe.cu): every CTA routes redundantly; the
// 2 x Hx hidden units, then the D x 2 down rows, are split evenly over the
// grid with one grid barrier between; a CTA requests its down rows (words and
// group scales, into registers) before the barrier.  A warp dots one row:
// lane l takes the row's 32-bit words l, l + 32, ... (4 int8 or 8 int4 values
// of one group, multiplied with x in fp32, the word's sum times the group
// scale added to the lane's total), so a warp's loads of weights are 128-byte
// coalesced and its reads of x in shared memory are conflict-free.
#include "kernels.h"
#include "stream.cuh"

namespace mie {

namespace {

constexpr int kQThreads = 512;
constexpr int kQWarps = kQThreads / 32;
constexpr int kQSegWords = 6;  // words per lane held in registers per row segment (a 768-element int8 row)

__device__ __forceinline__ float q_gelu(float v) { return 0.5f * v * (1.0f + erff(v * 0.7071067811865476f)); }
__device__ __forceinline__ float q_silu(float v) { return v / (1.0f + expf(-v)); }

// Elements per 32-bit word.
template <int BITS>
constexpr int kEpw = 32 / BITS;

// The lane's words of one segment (32 x kQSegWords words) of a quantized row,
// with the scale of each word's group.
template <int BITS>
struct QSeg {
  uint32_t q[kQSegWords];
  float s[kQSegWords];
};

// gsh = log2(group): the group of element i is i >> gsh (group a power of two)
template <int BITS>
__device__ __forceinline__ void qseg_load(QSeg<BITS>& r, const uint32_t* row, const float* scale, int nw, int gsh,
                                          int seg) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < kQSegWords; ++k) {
    const int w = seg * 32 * kQSegWords + lane + 32 * k;
    if (w < nw) {
      r.q[k] = __ldg(row + w);
      r.s[k] = __ldg(scale + ((w * kEpw<BITS>) >> gsh));
    }
  }
}


// sum over the segment's words of scale x (q . x); x fp32 in shared memory
template <int BITS>
__device__ __forceinline__ float qseg_dot(const QSeg<BITS>& r, const float* xs, int nw, int seg, float acc) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < kQSegWords; ++k) {
    const int w = seg * 32 * kQSegWords + lane + 32 * k;
    if (w < nw) {
      float part;
      if constexpr (BITS == 8) {
        const uint32_t u = r.q[k] ^ 0x80808080u;
        const float4 x = *reinterpret_cast<const float4*>(xs + 4 * w);
        // byte b to the low byte, zeros, 0x4B on top
        part = byte_to_f(u, 0x7440u) * x.x;
        part = fmaf(byte_to_f(u, 0x7441u), x.y, part);
        part = fmaf(byte_to_f(u, 0x7442u), x.z, part);
        part = fmaf(byte_to_f(u, 0x7443u), x.w, part);
      } else {
        const uint32_t u = r.q[k] ^ 0x88888888u;
        const float4 x0 = *reinterpret_cast<const float4*>(xs + 8 * w);
        const float4 x1 = *reinterpret_cast<const float4*>(xs + 8 * w + 4);
        const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        part = 0.f;
#pragma unroll
        for (int b = 0; b < 8; ++b) part = fmaf(nibble_to_f(u, b), xv[b], part);
      }
      acc = fmaf(r.s[k], part, acc);
    }
  }
  return acc;
}

// Full dot of one quantized row of n elements with xs (segment by segment).
template <int BITS>
__device__ __forceinline__ float qrow_dot(const uint32_t* row, const float* scale, const float* xs, int n, int gsh) {
  const int nw = n / kEpw<BITS>;
  const int nseg = (nw + 32 * kQSegWords - 1) / (32 * kQSegWords);
  float acc = 0.f;
  for (int sg = 0; sg < nseg; ++sg) {
    QSeg<BITS> r;
    qseg_load<BITS>(r, row, scale, nw, gsh, sg);
    acc = qseg_dot<BITS>(r, xs, nw, sg, acc);
  }
  return warp_sum(acc);
}

template <typename X, int BITS>
__global__ void __launch_bounds__(kQThreads) moe_decode_q_kernel(const mie_moe_args a, MoeLayout L) {
  extern __shared__ __align__(16) float smem_q[];
  const int D = a.hidden_dim, Hx = a.expert_hidden_dim, E = a.num_experts, grp = a.group_size;
  const int gsh = __ffs(grp) - 1;  // group_size is a power of two (checked on the host)
  const int G = gridDim.x, c = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool swiglu = a.act == MIE_ACT_SWIGLU;
  float* xs = smem_q;            // [D] normalised input
  float* hs = xs + L.off_h;      // [2, Hx] expert activations
  float* resD = xs + L.off_res;  // [2, max_rows] down-projection results
  __shared__ float red[kQWarps];
  __shared__ float logits_s[32];
  __shared__ int ids_s[2];
  __shared__ float wts_s[2];
  __shared__ uint64_t target_s;
  uint64_t* ctr = reinterpret_cast<uint64_t*>(a.sync);
  if (tid == 0) target_s = grid_sync_target(ctr, (uint32_t)G);
  // Router rows (in the activation type) are static: requested into registers
  // before waiting on the producer grid, dotted as the bf16 kernel does (the
  // same logits, so the same routing)
  constexpr int PV = Elem<X>::kPerVec;
  const int nvec_d = D / PV;
  const int64_t rb_d = (int64_t)D * sizeof(X);
  const bool r_regs = nvec_d <= Seg<X>::kVecs;
  auto router_row = [&](int e) {
    return reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.router_w) + e * rb_d);
  };
  RowRegs<X> rr[2];
  if (r_regs) {
    for (int k = 0; k < 2; ++k)
      if (warp + kQWarps * k < E) row_load<X>(rr[k], router_row(warp + kQWarps * k), nvec_d, 0);
  }

  pdl_wait();
  if (skip_requested(a.skip)) {
    pdl_trigger();
    return;
  }
  // expert parallel with the all-reduce fused in: this launch's call number
  __shared__ uint32_t ptag_s;
  const bool peer = a.peer_world > 1 && !L.route_only;
  if (peer && tid == 0) ptag_s = peer_tag(a);

  // ---- prologue: norm + router + top-2, every CTA ----
  load_and_norm(xs, a.x, a.x_dtype, nullptr, D, a.norm, a.eps, a.norm_w, a.norm_b, a.dtype, red);
  float xr[Seg<X>::kNV * PV];
  if (r_regs) load_x_regs<X>(xr, xs, nvec_d);
  for (int k = 0; k < 2; ++k) {
    const int e = warp + kQWarps * k;
    if (e < E) {
      const float v = r_regs ? warp_sum(row_dot_regs<X>(rr[k], xr)) : warp_row_dot<X>(router_row(e), nvec_d, xs);
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

  // ---- this CTA's work: up units [u0, u1), down rows [r0, r1) x 2 experts ----
  const int ebase = a.expert_base;
  const int ecount = a.expert_count > 0 ? a.expert_count : E;
  int u0, u1, r0, r1;
  split_range(2 * Hx, c, G, &u0, &u1);
  split_range(D, c, G, &r0, &r1);
  const int nu = u1 - u0, nr = r1 - r0, np = 2 * nr;
  int le[2];
  bool local[2];
  for (int r = 0; r < 2; ++r) {
    le[r] = ids_s[r] - ebase;
    local[r] = le[r] >= 0 && le[r] < ecount;
  }
  const int wpr_d = D / kEpw<BITS>, wpr_h = Hx / kEpw<BITS>;  // words per up row / per down row
  const int spr_d = D / grp, spr_h = Hx / grp;                // group scales per row
  const uint32_t* q1 = static_cast<const uint32_t*>(a.w1);
  const uint32_t* q3 = static_cast<const uint32_t*>(a.w3);
  const uint32_t* q2 = static_cast<const uint32_t*>(a.w2);
  const bool up_regs = wpr_d <= 32 * kQSegWords, dn_regs = wpr_h <= 32 * kQSegWords;

  // this warp's first down row, requested now (it depends on the routing only)
  QSeg<BITS> wd;
  if (dn_regs && warp < np && local[warp / nr]) {
    const int64_t row = (int64_t)le[warp / nr] * D + r0 + warp % nr;
    qseg_load<BITS>(wd, q2 + row * wpr_h, a.w2_scale + row * spr_h, wpr_h, gsh, 0);
  }

  // ---- up phase: unit k -> slot r = u / Hx, hidden index j ----
  for (int k = warp; k < nu; k += kQWarps) {
    const int u = u0 + k, r = u / Hx, j = u - r * Hx;
    if (!local[r]) continue;
    const int64_t row = (int64_t)le[r] * Hx + j;
    float g, uv = 0.f;
    if (up_regs) {
      QSeg<BITS> ga, ua;
      qseg_load<BITS>(ga, q1 + row * wpr_d, a.w1_scale + row * spr_d, wpr_d, gsh, 0);
      if (swiglu) qseg_load<BITS>(ua, q3 + row * wpr_d, a.w3_scale + row * spr_d, wpr_d, gsh, 0);
      g = warp_sum(qseg_dot<BITS>(ga, xs, wpr_d, 0, 0.f));
      if (swiglu) uv = warp_sum(qseg_dot<BITS>(ua, xs, wpr_d, 0, 0.f));
    } else {
      g = qrow_dot<BITS>(q1 + row * wpr_d, a.w1_scale + row * spr_d, xs, D, gsh);
      if (swiglu) uv = qrow_dot<BITS>(q3 + row * wpr_d, a.w3_scale + row * spr_d, xs, D, gsh);
    }
    if (lane == 0) {
      if (a.b1) g += load_any(a.b1, a.dtype, row);
      a.hidden[(int64_t)r * Hx + j] = swiglu ? q_silu(g) * uv : q_gelu(g);
    }
  }

  // ---- grid barrier: every CTA's h is in global memory ----
  const bool ok = grid_sync(ctr, target_s, a.status);
  pdl_trigger();
  if (!ok) return;
  for (int i = tid; i < 2 * Hx; i += blockDim.x) hs[i] = __ldcg(a.hidden + i);
  __syncthreads();

  // ---- down phase: pair p -> slot r = p / nr, output row r0 + p % nr ----
  for (int p = warp; p < np; p += kQWarps) {
    const int r = p / nr, rowi = r0 + p % nr;
    if (!local[r]) continue;
    const int64_t row = (int64_t)le[r] * D + rowi;
    float v;
    if (dn_regs) {
      if (p != warp) qseg_load<BITS>(wd, q2 + row * wpr_h, a.w2_scale + row * spr_h, wpr_h, gsh, 0);
      v = warp_sum(qseg_dot<BITS>(wd, hs + (size_t)r * Hx, wpr_h, 0, 0.f));
    } else {
      v = qrow_dot<BITS>(q2 + row * wpr_h, a.w2_scale + row * spr_h, hs + (size_t)r * Hx, Hx, gsh);
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

template <typename X>
void* pick_q(int bits) {
  return bits == 8 ? (void*)moe_decode_q_kernel<X, 8> : bits == 4 ? (void*)moe_decode_q_kernel<X, 4> : nullptr;
}

}  // namespace

int moe_decode_q_launch(const mie_moe_args& a, const MoeLayout& L, int grid, cudaStream_t st, bool pdl) {
  void* k = a.dtype == MIE_BF16 ? pick_q<__nv_bfloat16>(a.expert_bits) : pick_q<float>(a.expert_bits);
  if (!k) return MIE_ERR_UNSUPPORTED;
  using K = void (*)(const mie_moe_args, MoeLayout);
  return launch(reinterpret_cast<K>(k), dim3(grid), dim3(kQThreads), L.smem, st, pdl, a, L);
}

void moe_q_set_attributes() {
  for (int bits : {8, 4}) {
    set_max_smem(reinterpret_cast<void (*)(const mie_moe_args, MoeLayout)>(pick_q<__nv_bfloat16>(bits)));
    set_max_smem(reinterpret_cast<void (*)(const mie_moe_args, MoeLayout)>(pick_q<float>(bits)));
  }
}

}  // namespace mie
