// Row-chunk streaming for the M=1 GEMV kernels.
//
// Every GEMV here reads each weight row exactly once.  A CTA owns a list of
// "chunks" (runs of consecutive rows, contiguous in HBM); one thread moves each
// chunk into a shared-memory ring slot with cp.async.bulk (TMA bulk copy,
// completion counted in bytes on the slot's mbarrier) and all warps consume
// the slot (one warp per row, 16-byte vector loads from shared memory, a
// shuffle reduction per row).  Keeping `nslot` chunks in flight per SM hides
// HBM latency with a single issuing thread.
#pragma once

#include "common.cuh"

namespace mie {

struct Chunk {
  const uint8_t* src;  // first byte of the first row (16-byte aligned)
  uint32_t bytes;      // rows * row_bytes (multiple of 16)
  uint16_t rows;
  uint8_t tag;         // kernel-defined meaning
  uint8_t sub;         // kernel-defined (e.g. top-k slot)
  int32_t out;         // kernel-defined output index of the first row
};

struct Ring {
  uint64_t* bar;  // [nslot] mbarriers (count 1, tx-counted)
  uint8_t* data;  // nslot * slot_bytes, 128-byte aligned
  int nslot;
  uint32_t slot_bytes;
  __device__ __forceinline__ uint8_t* slot(int i) const { return data + (size_t)i * slot_bytes; }
};

// thread 0: initialise the ring's barriers (call before __syncthreads()).
__device__ __forceinline__ void ring_init(const Ring& R) {
  for (int s = 0; s < R.nslot; ++s) mbar_init(&R.bar[s], 1);
  fence_barrier_init();
}

// thread 0: start the copy of chunk i into slot i % nslot.
__device__ __forceinline__ void ring_issue(const Ring& R, const Chunk& c, int i, uint64_t policy) {
  const int s = i % R.nslot;
  uint64_t* bar = &R.bar[s];
  mbar_arrive_expect_tx(bar, c.bytes);
  uint8_t* dst = R.slot(s);
  for (uint32_t off = 0; off < c.bytes; off += kBulkMax) {
    const uint32_t n = (c.bytes - off) < kBulkMax ? (c.bytes - off) : kBulkMax;
    bulk_g2s_stream(dst + off, c.src + off, n, bar, policy);
  }
}

// thread 0: wait (bounded) for chunks [from, to) that were issued but will not
// be consumed, so no bulk copy is still writing shared memory at exit.
__device__ __forceinline__ void ring_drain(const Ring& R, int from, int to, int32_t* status) {
  for (int i = from; i < to; ++i) mbar_wait(&R.bar[i % R.nslot], (i / R.nslot) & 1, status);
}

// Consume chunks [0, n) in order.  `issued` chunks were started already
// (issued <= nslot); later ones are started as slots free up.  process(i,
// chunk, slot_ptr) is called by every thread.  Returns false if a wait gave up
// (after draining what is still in flight).
template <typename Process>
__device__ __forceinline__ bool ring_consume(const Ring& R, const Chunk* chunks, int n, int issued,
                                             uint64_t policy, int32_t* status, Process&& process) {
  for (int i = 0; i < n; ++i) {
    if (threadIdx.x == 0) {
      // Top up the ring: chunk i must have been issued before we wait on it.
      while (issued < n && issued < i + R.nslot) {
        if (issued >= R.nslot) fence_proxy_async_smem();
        ring_issue(R, chunks[issued], issued, policy);
        ++issued;
      }
    }
    const int s = i % R.nslot;
    const bool ok = mbar_wait(&R.bar[s], (i / R.nslot) & 1, status);
    if (!__syncthreads_and(ok)) {
      if (threadIdx.x == 0) ring_drain(R, i + 1, min(n, i + R.nslot), status);
      return false;
    }
    process(i, chunks[i], R.slot(s));
    __syncthreads();
  }
  return true;
}

// Dot every row of a chunk (rows x row_elems elements of W, row-major in
// shared memory) with the fp32 vector `vec` (shared memory).  One warp per row;
// emit(row, value) runs on lane 0 of the warp that owns the row.
template <typename W, typename Emit>
__device__ __forceinline__ void chunk_dot_rows(const uint8_t* slot, int rows, int row_elems,
                                               const float* __restrict__ vec, Emit&& emit) {
  constexpr int PV = Elem<W>::kPerVec;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int nvec = row_elems / PV;
  for (int r = warp; r < rows; r += nw) {
    const uint4* row = reinterpret_cast<const uint4*>(slot) + (size_t)r * nvec;
    float acc = 0.f;
    for (int v = lane; v < nvec; v += kWarp) acc = dot_vec(row[v], vec + v * PV, acc, (const W*)nullptr);
    acc = warp_sum(acc);
    if (lane == 0) emit(r, acc);
  }
}

// Split [begin, end) rows starting at `base` (row_bytes each) into chunks of
// at most `cap` rows, appending to chunks[*n].  Returns false on overflow.
__device__ __forceinline__ bool push_rows(Chunk* chunks, int* n, int max_chunks, const void* base,
                                          int64_t row_begin, int rows, uint32_t row_bytes, int cap,
                                          uint8_t tag, uint8_t sub, int32_t out) {
  const uint8_t* p = static_cast<const uint8_t*>(base) + row_begin * (int64_t)row_bytes;
  for (int r = 0; r < rows; r += cap) {
    if (*n >= max_chunks) return false;
    const int k = (rows - r) < cap ? (rows - r) : cap;
    Chunk c;
    c.src = p + (int64_t)r * row_bytes;
    c.bytes = (uint32_t)k * row_bytes;
    c.rows = (uint16_t)k;
    c.tag = tag;
    c.sub = sub;
    c.out = out + r;
    chunks[(*n)++] = c;
  }
  return true;
}

// Input-vector prologue shared by the QKV, MoE and LM-head kernels:
// xs[i] = (x[i] (+ add[i])) then optional RMSNorm / LayerNorm with weight w
// (and bias b).  Deterministic: every CTA computes bit-identical values.
// `red` needs blockDim.x/32 floats.
__device__ __forceinline__ void load_and_norm(float* xs, const void* x, int x_dtype, const float* add, int D,
                                              int norm, float eps, const void* w, const void* b, int w_dtype,
                                              float* red) {
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float v = load_any(x, x_dtype, i);
    if (add) v += add[i];
    xs[i] = v;
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

// Contiguous share of `total` items for CTA `c` of `g`: [begin, end).
__device__ __forceinline__ void split_range(int total, int c, int g, int* begin, int* end) {
  *begin = (int)(((int64_t)total * c) / g);
  *end = (int)(((int64_t)total * (c + 1)) / g);
}

}  // namespace mie
