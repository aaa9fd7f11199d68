// Register-staged row loads for the M=1 GEMV kernels.
//
// Every GEMV here reads each weight row exactly once.  A warp owns whole rows:
// lane l loads 16-byte vectors l, l+32, l+64, ... of a row with plain
// read-only 128-bit loads straight into registers, then forms the dot product
// with the fp32 input vector and reduces it with shuffles.  A warp issues the
// loads of several rows before it uses any of them, so each SM keeps tens of
// KB in flight without shared-memory staging, async-copy units or barriers.
// Rows whose weights do not depend on the producer grid are loaded before the
// kernel waits on it (programmatic dependent launch), i.e. while the previous
// kernel still runs.
//
// A row is processed in segments of 768 elements (3 vectors per lane for
// bf16, 6 for fp32); longer rows loop over segments.
#pragma once

#include <cstdio>

#include "common.cuh"
#include "exchange.cuh"

namespace mie {

// 16-byte vectors per lane per row segment (a segment = 768 elements).
template <typename W>
struct Seg {
  static constexpr int kNV = 768 / (kWarp * Elem<W>::kPerVec);  // bf16: 3, fp32: 6
  static constexpr int kVecs = kNV * kWarp;                      // vectors per segment
};

template <typename W>
struct RowRegs {
  uint4 w[Seg<W>::kNV];
};

__device__ __forceinline__ uint4 ld_weights(const uint4* p) { return __ldg(p); }

// Load segment `seg` of a row (nvec 16-byte vectors) into this lane's registers.
template <typename W>
__device__ __forceinline__ void row_load(RowRegs<W>& r, const uint4* row, int nvec, int seg) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < Seg<W>::kNV; ++j) {
    const int v = seg * Seg<W>::kVecs + lane + kWarp * j;
    r.w[j] = v < nvec ? ld_weights(row + v) : make_uint4(0u, 0u, 0u, 0u);
  }
}

// This lane's partial dot of a loaded segment with the fp32 vector xs (shared).
template <typename W>
__device__ __forceinline__ float row_dot(const RowRegs<W>& r, const float* __restrict__ xs, int nvec, int seg,
                                         float acc = 0.f) {
  constexpr int PV = Elem<W>::kPerVec;
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < Seg<W>::kNV; ++j) {
    const int v = seg * Seg<W>::kVecs + lane + kWarp * j;
    if (v < nvec) acc = dot_vec(r.w[j], xs + v * PV, acc, (const W*)nullptr);
  }
  return acc;
}

// Same with x already held in registers (segment 0 of xs, see load_x_regs).
template <typename W>
__device__ __forceinline__ float row_dot_regs(const RowRegs<W>& r, const float* xr) {
  constexpr int PV = Elem<W>::kPerVec;
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < Seg<W>::kNV; ++j) acc = dot_vec(r.w[j], xr + j * PV, acc, (const W*)nullptr);
  return acc;
}

// xr[j*PV + e] = xs[(lane + 32 j) * PV + e] for segment 0 (zero past nvec);
// xs 16-byte aligned in shared memory.  16-byte loads.  For bf16 rows a lane
// needs 32 bytes of x (two 16-byte halves); lanes 4-7 of every quarter-warp
// read their halves in the opposite order to lanes 0-3, so each 16-byte load
// instruction of a quarter-warp touches eight distinct bank groups (no bank
// conflicts; in natural order lanes i and i + 4 would collide).
template <typename W>
__device__ __forceinline__ void load_x_regs(float* xr, const float* xs, int nvec) {
  constexpr int PV = Elem<W>::kPerVec;
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < Seg<W>::kNV; ++j) {
    const int v = lane + kWarp * j;
    if constexpr (PV == 4) {
      const float4 a = v < nvec ? *reinterpret_cast<const float4*>(xs + v * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
      xr[j * 4 + 0] = a.x;
      xr[j * 4 + 1] = a.y;
      xr[j * 4 + 2] = a.z;
      xr[j * 4 + 3] = a.w;
    } else {
      const int h0 = (lane >> 2) & 1;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
      if (v < nvec) {
        a = *reinterpret_cast<const float4*>(xs + v * 8 + 4 * h0);
        b = *reinterpret_cast<const float4*>(xs + v * 8 + 4 * (1 - h0));
      }
      const float4 lo = h0 ? b : a, hi = h0 ? a : b;
      xr[j * 8 + 0] = lo.x;
      xr[j * 8 + 1] = lo.y;
      xr[j * 8 + 2] = lo.z;
      xr[j * 8 + 3] = lo.w;
      xr[j * 8 + 4] = hi.x;
      xr[j * 8 + 5] = hi.y;
      xr[j * 8 + 6] = hi.z;
      xr[j * 8 + 7] = hi.w;
    }
  }
}

// Full dot of one row with xs (any length), loads issued segment by segment.
template <typename W>
__device__ __forceinline__ float warp_row_dot(const uint4* row, int nvec, const float* xs) {
  const int nseg = (nvec + Seg<W>::kVecs - 1) / Seg<W>::kVecs;
  float acc = 0.f;
  for (int s = 0; s < nseg; ++s) {
    RowRegs<W> r;
    row_load<W>(r, row, nvec, s);
    acc = row_dot<W>(r, xs, nvec, s, acc);
  }
  return warp_sum(acc);
}

// Input-vector prologue shared by the QKV, MoE and LM-head kernels:
// xs[i] = (x[i] (+ add[i])) then optional RMSNorm / LayerNorm with weight w
// (and bias b).  x is a global pointer (read through L2: it was written by an
// earlier grid), or nullptr when xs already holds the input.  Deterministic:
// every CTA computes bit-identical values.  `red` needs blockDim.x/32 floats.
__device__ __forceinline__ void load_and_norm(float* xs, const void* x, int x_dtype, const float* add, int D,
                                              int norm, float eps, const void* w, const void* b, int w_dtype,
                                              float* red) {
  if (x) {
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
      float v = x_dtype == MIE_F32 ? __ldcg(static_cast<const float*>(x) + i) : load_any(x, x_dtype, i);
      if (add) v += __ldcg(add + i);
      xs[i] = v;
    }
  }
  __syncthreads();
  if (norm == MIE_NORM_RMS) {
    float ss = 0.f;
    for (int i = threadIdx.x; i < D; i += blockDim.x) ss = fmaf(xs[i], xs[i], ss);
    ss = block_sum(ss, red);
    const float r = rsqrtf(ss / (float)D + eps);
    for (int i = threadIdx.x; i < D; i += blockDim.x) xs[i] = (xs[i] * r) * load_any(w, w_dtype, i);
  } else if (norm == MIE_NORM_LAYER) {
    float s = 0.f;
    for (int i = threadIdx.x; i < D; i += blockDim.x) s += xs[i];
    const float mean = block_sum(s, red) / (float)D;
    float v = 0.f;
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
      const float d = xs[i] - mean;
      v = fmaf(d, d, v);
    }
    const float var = block_sum(v, red) / (float)D;
    const float r = rsqrtf(var + eps);
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
      float y = (xs[i] - mean) * r * load_any(w, w_dtype, i);
      if (b) y += load_any(b, w_dtype, i);
      xs[i] = y;
    }
  }
  __syncthreads();
}

// Top-2 of E logits by repeated argmax -- a strict '>' while scanning
// ascending ids keeps the lower id on ties (fused_moe.py:146-150) -- and the
// stable 2-way softmax of the pair (l0 >= l1).
__device__ __forceinline__ void top2_route(const float* logits, int E, int* id0, int* id1, float* w0, float* w1) {
  int i0 = 0;
  for (int e = 1; e < E; ++e)
    if (logits[e] > logits[i0]) i0 = e;
  int i1 = (i0 == 0) ? 1 : 0;
  for (int e = 0; e < E; ++e)
    if (e != i0 && logits[e] > logits[i1]) i1 = e;
  const float e1 = expf(logits[i1] - logits[i0]);
  const float den = 1.0f + e1;
  *id0 = i0;
  *id1 = i1;
  *w0 = 1.0f / den;
  *w1 = e1 / den;
}

// Expert parallel with the all-reduce fused into the MoE kernels (the
// peer_* fields of mie_moe_args; the exchange of mie_peer_reduce, done by the
// CTA that owns the rows).  peer_tag: this launch's call number, read after
// the dependency wait and before the grid barrier (CTA 0 advances the counter
// after it).  peer_row_sum: row `row` of this rank's partial y into every
// rank's receive buffer, then the rank-order sum of that row over the ranks;
// a wait that runs out records MIE_ERR_TIMEOUT and returns y.
__device__ __forceinline__ uint32_t peer_tag(const mie_moe_args& a) {
  return *reinterpret_cast<volatile const uint32_t*>(a.peer_seq) + 1u;
}
__device__ __forceinline__ float peer_row_sum(const mie_moe_args& a, int D, int row, float y, uint32_t tag) {
  const size_t half = (size_t)(tag & 1u) * (size_t)a.peer_world * D;
  for (int r = 0; r < a.peer_world; ++r) ll_put_sys(a.peer_bufs[r] + half + (size_t)a.peer_rank * D + row, y, tag);
  const uint64_t* mine = a.peer_bufs[a.peer_rank] + half + row;
  const unsigned long long limit = a.peer_wait_limit_ns > 0 ? (unsigned long long)a.peer_wait_limit_ns : kWaitLimitNs;
  float sum = 0.f;
  for (int r = 0; r < a.peer_world; ++r) {
    const uint64_t* p = mine + (size_t)r * D;
    uint64_t w = ll_ld_sys(p);
    if (ll_tag(w) != tag) {
      const unsigned long long t0 = global_ns();
      while (ll_tag(w = ll_ld_sys(p)) != tag) {
        if (global_ns() - t0 > limit) {
          set_status(a.status, MIE_ERR_TIMEOUT);
          return y;
        }
      }
    }
    sum += ll_val(w);
  }
  return sum;
}

// Small integers to float without I2F: with the bit pattern 0x4B000000 | u
// (u < 2^23) a float holds exactly 2^23 + u, so subtracting 2^23 + bias
// leaves u - bias.  Quantized expert values are offset to unsigned (q + 128
// for int8, q + 8 for int4) by flipping their sign bits when loaded.
__device__ __forceinline__ float byte_to_f(uint32_t u_flipped, uint32_t sel) {
  return __int_as_float(__byte_perm(u_flipped, 0x4B000000u, sel)) - 8388736.0f;  // 2^23 + 128
}
__device__ __forceinline__ float nibble_to_f(uint32_t u_flipped, int b) {
  return __int_as_float(0x4B000000u | ((u_flipped >> (4 * b)) & 0xFu)) - 8388616.0f;  // 2^23 + 8
}

// Contiguous share of `total` items for CTA `c` of `g`: [begin, end).
__device__ __forceinline__ void split_range(int total, int c, int g, int* begin, int* end) {
  *begin = (int)(((int64_t)total * c) / g);
  *end = (int)(((int64_t)total * (c + 1)) / g);
}

}  // namespace mie
