// Single-query (decode) attention over a paged or contiguous K/V cache, sm_100a.
//
// Reference: src/moe_engine/paged_attention.py:47-154 (one Triton program per
// head looping over 128-token tiles with an online softmax) and the contiguous
// SDPA decode at src/moe_engine/model.py:261-266.
//
// Here the context of every head is split over `splits` CTAs (grid = splits x
// heads) so all SMs stream K/V.  A CTA walks its token range in stages of up
// to 32 KB of K+V: every thread loads its 16-byte pieces of the stage with
// plain read-only loads into registers (a block of one head is bs*hd
// contiguous elements in the [nb, H, bs, hd] pool; the contiguous [H, S, hd]
// layout is the same addressing with an identity block map), stores them to
// one of two shared-memory buffers, and the next stage's loads are in flight
// while the current stage is reduced.  An online softmax (running max m,
// normaliser l, accumulator acc) gives the CTA's (m, l, acc).  The last CTA of
// each head (arrival counter, no spinning) merges the partials with a
// log-sum-exp rescale and writes the output row -- or, with defer_merge, the
// consumer kernel merges them (the decode step's out_proj).
//
// Under programmatic dependent launch the stages that hold only OLD tokens are
// loaded before waiting on the producer grid (the QKV kernel that writes the
// newest token); the stage holding the newest token is loaded after.
#include <mutex>
#include <utility>

#include "kernels.h"
#include "stream.cuh"

namespace mie {

namespace {

constexpr int kThreads = 128;
constexpr int kStageVecs = 16;  // 16-byte K/V pieces per thread per stage (32 KB per CTA)

template <typename KV, int HD>
__global__ void __launch_bounds__(kThreads) attn_decode_kernel(const mie_attn_args a, AttnLayout L) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int h = blockIdx.y, s = blockIdx.x, S = gridDim.x, tid = threadIdx.x;
  const int bs = a.block_size;
  KV* kvbuf = reinterpret_cast<KV*>(smem + L.off_kv);
  float* q_s = reinterpret_cast<float*>(smem + L.off_q);
  float* p_s = reinterpret_cast<float*>(smem + L.off_p);
  float* acc_s = reinterpret_cast<float*>(smem + L.off_acc);
  __shared__ float red[kThreads / 32];
  __shared__ int last_s;
  const int stage_tok = L.stage_tokens;
  const int stage_blocks = stage_tok / bs;
  const size_t stage_elems = (size_t)2 * stage_tok * HD;  // K then V
  constexpr bool kVec = (HD * sizeof(KV)) % 16 == 0;
  constexpr int VPT = kVec ? 16 / (int)sizeof(KV) : 1;  // elements per 16-byte piece
  constexpr int VPH = kVec ? HD / VPT : 1;              // pieces per head row

  // Context length.  ctx_dev is the step's device position, written by an
  // earlier step's LM-head kernel that completed before this grid's producer
  // started, so it may be read before pdl_wait().  Out-of-range values are
  // clamped here and reported only after the skip flag was read (a skipped
  // step may carry a stale position).
  int ctx = a.ctx_dev ? (__ldcg(a.ctx_dev) + a.ctx_dev_offset) : a.ctx_len;
  const bool bad_ctx = ctx < 1 || ctx > a.max_ctx;
  if (bad_ctx) ctx = ctx < 1 ? 1 : a.max_ctx;
  const int nblk = (ctx + bs - 1) / bs;
  int b0, b1;
  split_range(nblk, s, S, &b0, &b1);
  const int nst = (b1 - b0 + stage_blocks - 1) / stage_blocks;
  // The stage holding the newest token (always this CTA's last stage) is
  // loaded only after the producer grid finished.
  const int nst_pre = (a.new_token_last && b1 == nblk && nst > 0) ? nst - 1 : nst;

  auto phys_of = [&](int b) -> int64_t {
    if (!a.block_table) return b;
    int p = __ldg(a.block_table + b);
    if (p < 0 || p >= a.num_blocks) {
      set_status(a.status, MIE_ERR_RANGE);
      p = 0;
    }
    return p;
  };
  auto tile_ptr = [&](const void* base, int64_t phys) {
    return static_cast<const KV*>(base) + phys * a.stride_block + (int64_t)h * a.stride_head;
  };
  auto stage_tokens = [&](int st) {
    const int bb = b0 + st * stage_blocks, be = min(b1, bb + stage_blocks);
    return min(be * bs, ctx) - bb * bs;
  };
  // Piece i of stage st: K pieces [0, n), then V pieces [n, 2n), n = tokens x VPH.
  auto piece_src = [&](int st, int i, int n) -> const uint4* {
    const int kv = i >= n, i2 = i - kv * n, t = i2 / VPH, sub = i2 - t * VPH;
    const int tok = (b0 + st * stage_blocks) * bs + t;
    const KV* base = tile_ptr(kv ? a.v : a.k, phys_of(tok / bs)) + (int64_t)(tok % bs) * a.stride_tok;
    return reinterpret_cast<const uint4*>(base + sub * VPT);
  };
  auto piece_dst = [&](int st, int i, int n) -> uint4* {
    const int kv = i >= n, i2 = i - kv * n, t = i2 / VPH, sub = i2 - t * VPH;
    KV* dst = kvbuf + (size_t)(st & 1) * stage_elems + (size_t)kv * stage_tok * HD + (size_t)t * HD + sub * VPT;
    return reinterpret_cast<uint4*>(dst);
  };
  uint4 pend[kStageVecs];
  auto stage_load = [&](int st) {  // registers <- global
    const int n = stage_tokens(st) * VPH;
#pragma unroll
    for (int m = 0; m < kStageVecs; ++m) {
      const int i = tid + kThreads * m;
      if (i < 2 * n) pend[m] = __ldg(piece_src(st, i, n));
    }
  };
  auto stage_store = [&](int st) {  // shared <- registers
    const int n = stage_tokens(st) * VPH;
#pragma unroll
    for (int m = 0; m < kStageVecs; ++m) {
      const int i = tid + kThreads * m;
      if (i < 2 * n) *piece_dst(st, i, n) = pend[m];
    }
  };

  int stored = 0;  // stages [0, stored) are in shared memory
  if constexpr (kVec) {
    for (; stored < min(2, nst_pre); ++stored) {
      stage_load(stored);
      stage_store(stored);
    }
  }

  pdl_wait();
  if (skip_requested(a.skip)) {
    pdl_trigger();
    return;
  }
  pdl_trigger();
  if (bad_ctx && tid == 0 && s == 0) set_status(a.status, MIE_ERR_RANGE);

  const float scale = a.scale;
  for (int d = tid; d < HD; d += kThreads) q_s[d] = load_any(a.q, a.q_dtype, (int64_t)h * HD + d);

  constexpr int G = kThreads / HD > 0 ? kThreads / HD : 1;  // PV token groups
  const int g = tid / HD, dcol = tid % HD;
  const bool pv_active = tid < G * HD;
  float acc = 0.f, m_run = -INFINITY, l_run = 0.f;

  for (int st = 0; st < nst; ++st) {
    const int bb = b0 + st * stage_blocks;
    const int t0 = bb * bs, ntok = stage_tokens(st);
    const KV* kst = kvbuf + (size_t)(st & 1) * stage_elems;
    const KV* vst = kst + (size_t)stage_tok * HD;
    bool pending = false;
    if constexpr (kVec) {
      if (stored == st) {  // not staged yet (the newest-token stage, or 1-buffer lag)
        stage_load(st);
        stage_store(st);
        ++stored;
      }
      __syncthreads();
      if (stored == st + 1 && st + 1 < nst) {  // next stage in flight while this one is reduced
        stage_load(st + 1);
        pending = true;
      }
    } else {
      // Rows too narrow for 16-byte pieces: element loads.
      KV* kw = const_cast<KV*>(kst);
      KV* vw = const_cast<KV*>(vst);
      __syncthreads();
      for (int i = tid; i < ntok * HD; i += kThreads) {
        const int t = i / HD, d = i % HD, b = (t0 + t) / bs, slot = (t0 + t) % bs;
        const int64_t p = phys_of(b);
        kw[i] = tile_ptr(a.k, p)[(int64_t)slot * a.stride_tok + d];
        vw[i] = tile_ptr(a.v, p)[(int64_t)slot * a.stride_tok + d];
      }
      __syncthreads();
    }

    // scores
    float mloc = -INFINITY;
    for (int t = tid; t < ntok; t += kThreads) {
      float dot = 0.f;
      if constexpr (kVec) {
        const uint4* kr = reinterpret_cast<const uint4*>(kst + (size_t)t * HD);
#pragma unroll
        for (int j = 0; j < VPH; ++j) {
          const int v = (j + t) % VPH;  // rotate the start piece: spreads banks
          dot = dot_vec(kr[v], q_s + v * VPT, dot, (const KV*)nullptr);
        }
      } else {
#pragma unroll
        for (int d = 0; d < HD; ++d) dot = fmaf(Elem<KV>::to_f(kst[(size_t)t * HD + d]), q_s[d], dot);
      }
      const float sc = dot * scale;
      p_s[t] = sc;
      mloc = fmaxf(mloc, sc);
    }
    const float m_stage = block_max(mloc, red);
    const float m_new = fmaxf(m_run, m_stage);
    const float alpha = (m_run == -INFINITY) ? 0.f : expf(m_run - m_new);
    float lsum = 0.f;
    for (int t = tid; t < ntok; t += kThreads) {
      const float p = expf(p_s[t] - m_new);
      p_s[t] = p;
      lsum += p;
    }
    const float l_stage = block_sum(lsum, red);  // ends with p_s visible to all
    l_run = l_run * alpha + l_stage;
    m_run = m_new;
    if (pv_active) {
      acc *= alpha;
      for (int t = g; t < ntok; t += G) acc = fmaf(p_s[t], Elem<KV>::to_f(vst[(size_t)t * HD + dcol]), acc);
    }
    __syncthreads();  // buffer (st + 1) & 1 == (st - 1) & 1 is no longer read
    if (pending) {
      stage_store(st + 1);
      ++stored;
    }
  }

  // combine the PV token groups
  if (pv_active) acc_s[g * HD + dcol] = acc;
  __syncthreads();
  const bool direct_out = (S == 1 && !a.defer_merge);
  float* part = a.partials + ((size_t)h * a.max_splits + s) * (HD + 2);
  for (int d = tid; d < HD; d += kThreads) {
    float v = 0.f;
    for (int gg = 0; gg < G; ++gg) v += acc_s[gg * HD + d];
    if (direct_out)
      store_any(a.out, a.out_dtype, (int64_t)h * HD + d, v / l_run);
    else
      part[2 + d] = v;
  }
  if (direct_out) return;
  if (tid == 0) {
    part[0] = m_run;
    part[1] = l_run;
  }
  if (a.defer_merge) return;
  __threadfence();
  __syncthreads();
  if (tid == 0) last_s = (atom_add_acq_rel_gpu(a.counters + h, 1u) == (uint32_t)(S - 1));
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  // log-sum-exp merge of the S partials of this head.  The partials are first
  // copied into shared memory (the K/V buffers are free) with every thread's
  // loads in flight together -- loaded one after another from L2 inside the
  // merge loops they made the merge a chain of dependent L2 round trips.
  const float* hp = a.partials + (size_t)h * a.max_splits * (HD + 2);
  float* ps = reinterpret_cast<float*>(kvbuf);  // [S][HD + 2]
  const int np = S * (HD + 2);
#pragma unroll 1
  for (int i0 = tid; i0 < np; i0 += 8 * kThreads) {
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i = i0 + k * kThreads;
      v[k] = i < np ? __ldcg(hp + i) : 0.f;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i = i0 + k * kThreads;
      if (i < np) ps[i] = v[k];
    }
  }
  __syncthreads();
  float M = -INFINITY;
  for (int j = 0; j < S; ++j) M = fmaxf(M, ps[j * (HD + 2)]);
  float Lsum = 0.f;
  for (int j = 0; j < S; ++j) {
    const float mj = ps[j * (HD + 2)];
    if (mj != -INFINITY) Lsum += ps[j * (HD + 2) + 1] * expf(mj - M);
  }
  for (int d = tid; d < HD; d += kThreads) {
    float o = 0.f;
    for (int j = 0; j < S; ++j) {
      const float mj = ps[j * (HD + 2)];
      if (mj != -INFINITY) o += ps[j * (HD + 2) + 2 + d] * expf(mj - M);
    }
    store_any(a.out, a.out_dtype, (int64_t)h * HD + d, o / Lsum);
  }
  if (tid == 0) a.counters[h] = 0u;  // ready for the next launch
}

// ---------------------------------------------------------------------------
// The cp.async kernel (rows of whole 16-byte pieces; the kernel above keeps
// the narrow rows).  256 threads; the split's physical block ids are read into
// shared memory first (one round trip instead of one per piece), then every
// thread issues 16-byte cp.async copies of the split's K and V rows into two
// chunk buffers of up to 48 KB each -- a split of up to two chunks has its
// whole range in flight at once -- and the chunks are reduced in order, a
// chunk's buffer refilled with the chunk after next once it is read.  Chunks
// holding only old tokens are issued before the programmatic-dependent wait.
// ---------------------------------------------------------------------------
constexpr int kFastThreads = 256;
constexpr uint32_t kFastChunkBytes = 48 * 1024;  // K + V of one chunk buffer

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <typename KV, int HD>
__global__ void __launch_bounds__(kFastThreads) attn_fast_kernel(const mie_attn_args a, AttnLayout L) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int T = kFastThreads;
  constexpr int VPT = 16 / (int)sizeof(KV), VPH = HD / VPT;  // 16-byte pieces per row
  constexpr int G = T / HD;                                   // PV token groups
  const int h = blockIdx.y, s = blockIdx.x, S = gridDim.x, tid = threadIdx.x;
  const int bs = a.block_size, chunk = L.chunk_tok;
  int* blk_s = reinterpret_cast<int*>(smem + L.off_blk);
  KV* kvb = reinterpret_cast<KV*>(smem + L.off_kv);  // [2 buffers][K | V][chunk][HD]
  float* q_s = reinterpret_cast<float*>(smem + L.off_q);
  float* sc = reinterpret_cast<float*>(smem + L.off_p);
  float* pv = reinterpret_cast<float*>(smem + L.off_acc);
  __shared__ float red[T / 32];
  __shared__ int last_s;

  // context length (see the kernel above: the device position may be read
  // before the dependency wait; out-of-range values are clamped, reported later)
  int ctx = a.ctx_dev ? (__ldcg(a.ctx_dev) + a.ctx_dev_offset) : a.ctx_len;
  const bool bad_ctx = ctx < 1 || ctx > a.max_ctx;
  if (bad_ctx) ctx = ctx < 1 ? 1 : a.max_ctx;
  const int nblk = (ctx + bs - 1) / bs;
  int b0, b1;
  split_range(nblk, s, S, &b0, &b1);
  const int tok0 = b0 * bs, tok1 = min(b1 * bs, ctx), ntok = max(0, tok1 - tok0);
  const int nch = (ntok + chunk - 1) / chunk;
  for (int i = tid; i < b1 - b0 && i < L.cap_blocks; i += T) {
    int p = b0 + i;  // contiguous cache: the identity block map
    if (a.block_table) {
      p = __ldg(a.block_table + b0 + i);
      if (p < 0 || p >= a.num_blocks) {
        set_status(a.status, MIE_ERR_RANGE);
        p = 0;
      }
    }
    blk_s[i] = p;
  }
  __syncthreads();
  auto issue = [&](int c) {  // chunk c -> buffer c & 1 (every thread; one commit group)
    const int t0 = tok0 + c * chunk, n = min(chunk, tok1 - t0);
    KV* kd = kvb + (size_t)(c & 1) * 2 * chunk * HD;
    KV* vd = kd + (size_t)chunk * HD;
    for (int j = tid; j < 2 * n * VPH; j += T) {
      const int v = j >= n * VPH, jj = j - v * n * VPH, t = jj / VPH, pc = jj - t * VPH;
      const int tok = t0 + t;
      const int64_t blk = blk_s[min(tok / bs - b0, L.cap_blocks - 1)];
      const KV* src = static_cast<const KV*>(v ? a.v : a.k) + blk * a.stride_block + (int64_t)h * a.stride_head +
                      (int64_t)(tok % bs) * a.stride_tok + pc * VPT;
      cp_async16((v ? vd : kd) + (size_t)t * HD + pc * VPT, src);
    }
    cp_async_commit();
  };
  // the split's last chunk holds the newest token when the producer grid
  // writes it: issued only after the wait
  const int nch_pre = (a.new_token_last && b1 == nblk && nch > 0) ? nch - 1 : nch;
  int issued = 0;
  for (; issued < min(2, nch_pre); ++issued) issue(issued);

  pdl_wait();
  if (skip_requested(a.skip)) {
    cp_async_wait<0>();  // nothing lands after the CTA left
    pdl_trigger();
    return;
  }
  pdl_trigger();
  if (bad_ctx && tid == 0 && s == 0) set_status(a.status, MIE_ERR_RANGE);
  for (; issued < min(2, nch); ++issued) issue(issued);
  for (int d = tid; d < HD; d += T) q_s[d] = load_any(a.q, a.q_dtype, (int64_t)h * HD + d);

  const float scale = a.scale;
  const int g = tid / HD, dcol = tid % HD;
  float acc = 0.f, m_run = -INFINITY, l_run = 0.f;
  for (int c = 0; c < nch; ++c) {
    if (issued - c - 1 >= 1)
      cp_async_wait<1>();
    else
      cp_async_wait<0>();
    __syncthreads();  // chunk c visible to every thread (and q_s)
    const int n = min(chunk, tok1 - (tok0 + c * chunk));
    const KV* kst = kvb + (size_t)(c & 1) * 2 * chunk * HD;
    const KV* vst = kst + (size_t)chunk * HD;
    float mloc = -INFINITY;
    for (int t = tid; t < n; t += T) {
      const uint4* kr = reinterpret_cast<const uint4*>(kst + (size_t)t * HD);
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < VPH; ++j) {
        const int v = (j + t) % VPH;  // rotate the start piece: spreads banks
        dot = dot_vec(kr[v], q_s + v * VPT, dot, (const KV*)nullptr);
      }
      const float scv = dot * scale;
      sc[t] = scv;
      mloc = fmaxf(mloc, scv);
    }
    const float m_new = fmaxf(m_run, block_max(mloc, red));
    const float alpha = (m_run == -INFINITY) ? 0.f : expf(m_run - m_new);
    float lsum = 0.f;
    for (int t = tid; t < n; t += T) {
      const float p = expf(sc[t] - m_new);
      sc[t] = p;
      lsum += p;
    }
    l_run = l_run * alpha + block_sum(lsum, red);  // ends with sc visible to all
    m_run = m_new;
    float a0 = 0.f, a1 = 0.f;
    int t = g;
    for (; t + G < n; t += 2 * G) {
      a0 = fmaf(sc[t], Elem<KV>::to_f(vst[(size_t)t * HD + dcol]), a0);
      a1 = fmaf(sc[t + G], Elem<KV>::to_f(vst[(size_t)(t + G) * HD + dcol]), a1);
    }
    if (t < n) a0 = fmaf(sc[t], Elem<KV>::to_f(vst[(size_t)t * HD + dcol]), a0);
    acc = fmaf(acc, alpha, a0 + a1);
    __syncthreads();  // buffer c & 1 and the scores are no longer read
    if (issued < nch) {
      issue(issued);
      ++issued;
    }
  }

  // combine the PV token groups
  pv[g * HD + dcol] = acc;
  __syncthreads();
  const bool direct_out = (S == 1 && !a.defer_merge);
  float* part = a.partials + ((size_t)h * a.max_splits + s) * (HD + 2);
  for (int d = tid; d < HD; d += T) {
    float v = 0.f;
#pragma unroll
    for (int gg = 0; gg < G; ++gg) v += pv[gg * HD + d];
    if (direct_out)
      store_any(a.out, a.out_dtype, (int64_t)h * HD + d, ntok > 0 ? v / l_run : 0.f);
    else
      part[2 + d] = v;
  }
  if (direct_out) return;
  if (tid == 0) {
    part[0] = m_run;
    part[1] = l_run;
  }
  if (a.defer_merge) return;
  __threadfence();
  __syncthreads();
  if (tid == 0) last_s = (atom_add_acq_rel_gpu(a.counters + h, 1u) == (uint32_t)(S - 1));
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  // log-sum-exp merge of the S partials of this head, staged in shared memory
  // (the chunk buffers are free) with every thread's loads in flight together
  const float* hp = a.partials + (size_t)h * a.max_splits * (HD + 2);
  float* ps = reinterpret_cast<float*>(kvb);  // [S][HD + 2]
  const int np = S * (HD + 2);
  for (int i0 = tid; i0 < np; i0 += 8 * T) {
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i = i0 + k * T;
      v[k] = i < np ? __ldcg(hp + i) : 0.f;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i = i0 + k * T;
      if (i < np) ps[i] = v[k];
    }
  }
  __syncthreads();
  float M = -INFINITY;
  for (int j = 0; j < S; ++j) M = fmaxf(M, ps[j * (HD + 2)]);
  float Lsum = 0.f;
  for (int j = 0; j < S; ++j) {
    const float mj = ps[j * (HD + 2)];
    if (mj != -INFINITY) Lsum += ps[j * (HD + 2) + 1] * expf(mj - M);
  }
  for (int d = tid; d < HD; d += T) {
    float o = 0.f;
    for (int j = 0; j < S; ++j) {
      const float mj = ps[j * (HD + 2)];
      if (mj != -INFINITY) o += ps[j * (HD + 2) + 2 + d] * expf(mj - M);
    }
    store_any(a.out, a.out_dtype, (int64_t)h * HD + d, o / Lsum);
  }
  if (tid == 0) a.counters[h] = 0u;  // ready for the next launch
}

// The cp.async kernel exists for rows of whole 16-byte pieces only.
template <typename KV, int HD>
void* fast_kernel_or_null() {
  if constexpr ((HD * sizeof(KV)) % 16 == 0)
    return (void*)attn_fast_kernel<KV, HD>;
  else
    return nullptr;
}
template <typename KV>
void* pick_fast(int hd) {
  switch (hd) {
    case 4: return fast_kernel_or_null<KV, 4>();
    case 8: return fast_kernel_or_null<KV, 8>();
    case 16: return fast_kernel_or_null<KV, 16>();
    case 32: return fast_kernel_or_null<KV, 32>();
    case 64: return fast_kernel_or_null<KV, 64>();
    case 96: return fast_kernel_or_null<KV, 96>();
    case 128: return fast_kernel_or_null<KV, 128>();
    default: return nullptr;
  }
}

template <typename KV>
void* pick(int hd) {
  switch (hd) {
    case 4: return (void*)attn_decode_kernel<KV, 4>;
    case 8: return (void*)attn_decode_kernel<KV, 8>;
    case 16: return (void*)attn_decode_kernel<KV, 16>;
    case 32: return (void*)attn_decode_kernel<KV, 32>;
    case 64: return (void*)attn_decode_kernel<KV, 64>;
    case 96: return (void*)attn_decode_kernel<KV, 96>;
    case 128: return (void*)attn_decode_kernel<KV, 128>;
    default: return nullptr;
  }
}

}  // namespace

AttnLayout attn_layout(const mie_attn_args& a) {
  const int esz = a.kv_dtype == MIE_BF16 ? 2 : 4;
  AttnLayout L{};
  // A stage (K+V) fits the threads' register staging: kStageVecs x 16 B per
  // thread; a whole number of blocks, at least one (narrow rows load per
  // element and are not limited by it).
  const int per_tok = 2 * a.head_dim * esz;
  const int budget = kStageVecs * 16 * kThreads;
  int st = (budget / per_tok) / a.block_size * a.block_size;
  if (st < a.block_size) st = a.block_size;
  L.stage_tokens = st;
  L.nstage = 2;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    off = (off + 127) & ~size_t(127);
    const size_t at = off;
    off += bytes;
    return (uint32_t)at;
  };
  L.off_bar = take(16);
  L.off_kv = take((size_t)L.nstage * per_tok * st);
  L.off_q = take(sizeof(float) * a.head_dim);
  L.off_p = take(sizeof(float) * st);
  L.off_acc = take(sizeof(float) * (kThreads > a.head_dim ? kThreads : a.head_dim));
  L.smem = (uint32_t)((off + 127) & ~size_t(127));
  // One block of K+V must fit the per-thread register staging (16-byte rows).
  if ((a.head_dim * esz) % 16 == 0 && per_tok * st > budget) L.smem = 0xffffffffu;  // -> unsupported
  // 16-byte rows run the cp.async kernel: two chunk buffers of up to 48 KB of
  // K + V each (whole blocks), the split's block ids, q, scores, PV partials
  if ((a.head_dim * esz) % 16 == 0 && a.splits > 0) {
    AttnLayout F{};
    F.fast = 1;
    int ct = (int)(kFastChunkBytes / (uint32_t)per_tok) / a.block_size * a.block_size;
    if (ct < a.block_size) ct = a.block_size;
    F.chunk_tok = ct;
    const int max_blk = (a.max_ctx + a.block_size - 1) / a.block_size;
    F.cap_blocks = (max_blk + a.splits - 1) / a.splits;
    if (F.cap_blocks < 1) F.cap_blocks = 1;
    off = 0;
    F.off_kv = take((size_t)2 * per_tok * ct);
    F.off_blk = take(sizeof(int) * (size_t)F.cap_blocks);
    F.off_q = take(sizeof(float) * a.head_dim);
    F.off_p = take(sizeof(float) * ct);
    F.off_acc = take(sizeof(float) * kFastThreads);
    F.smem = (uint32_t)((off + 127) & ~size_t(127));
    // the merge stages every split's partial in the chunk buffers
    if ((size_t)a.splits * (a.head_dim + 2) * 4 <= (size_t)2 * per_tok * ct && F.smem <= (uint32_t)kMaxDynSmem)
      return F;
  }
  return L;
}

int attn_decode_launch(const mie_attn_args& a, const AttnLayout& L, cudaStream_t st, bool pdl) {
  void* k = L.fast ? (a.kv_dtype == MIE_BF16 ? pick_fast<__nv_bfloat16>(a.head_dim) : pick_fast<float>(a.head_dim))
                   : (a.kv_dtype == MIE_BF16 ? pick<__nv_bfloat16>(a.head_dim) : pick<float>(a.head_dim));
  if (!k) return MIE_ERR_UNSUPPORTED;
  using K = void (*)(const mie_attn_args, AttnLayout);
  return launch(reinterpret_cast<K>(k), dim3(a.splits, a.num_heads), dim3(L.fast ? kFastThreads : kThreads), L.smem,
                st, pdl, a, L);
}

void attn_set_attributes() {
  for (int hd : {4, 8, 16, 32, 64, 96, 128}) {
    set_max_smem(pick<float>(hd));
    set_max_smem(pick<__nv_bfloat16>(hd));
    if (void* f = pick_fast<float>(hd)) set_max_smem(reinterpret_cast<void (*)(const mie_attn_args, AttnLayout)>(f));
    if (void* f = pick_fast<__nv_bfloat16>(hd))
      set_max_smem(reinterpret_cast<void (*)(const mie_attn_args, AttnLayout)>(f));
  }
}

// ---------------------------------------------------------------------------
// Fixed-scratch variant (mie_attn_decode_fixed_scratch)
//
// Some callers cannot allocate device memory: a host runtime that owns every
// byte of device memory and offers its plugins no allocator, or a
// latency-critical caller for which a cudaMalloc / cudaFree (which may
// synchronise the device) is not acceptable.  For them the split partials and
// the per-head merge counters live in this file-scope array instead of in
// caller-provided buffers.  Every GPU that loads the library holds it until
// the process exits.
//
// Layout (32-bit words): [0, kFixedCounters) merge counters, then
// kFixedPartialFloats floats of partials (num_heads x splits x (head_dim + 2)).
// ---------------------------------------------------------------------------
namespace {

constexpr int kFixedCounters = 64;                      // max heads
constexpr int kFixedPartialFloats = 64 * 1024;          // 256 KB of partials
constexpr int kFixedWords = kFixedCounters + kFixedPartialFloats;

static __device__ __align__(256) uint32_t g_attn_fixed_scratch[kFixedWords];

std::mutex g_fixed_mutex;
void* g_fixed_addr[64] = {nullptr};  // device address of the array, per device

// Once per device, with that device current: resolve the array's device
// address (the host symbol is only a stand-in) and zero the counters on the
// caller's stream, so the clear is ordered before this call's launch whatever
// kind of stream the caller uses.
int fixed_scratch_setup(void** out, cudaStream_t st) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    note_cuda_error(e, "cudaGetDevice");
    return MIE_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_fixed_mutex);
  if (!g_fixed_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_fixed_scratch);
    if (e != cudaSuccess) {
      note_cuda_error(e, "cudaGetSymbolAddress(g_attn_fixed_scratch)");
      return MIE_ERR_CUDA;
    }
    e = cudaMemsetAsync(p, 0, sizeof(uint32_t) * kFixedCounters, st);
    if (e != cudaSuccess) {
      note_cuda_error(e, "cudaMemsetAsync(fixed-scratch counters)");
      return MIE_ERR_CUDA;
    }
    g_fixed_addr[dev] = p;
  }
  *out = g_fixed_addr[dev];
  return MIE_OK;
}

}  // namespace

// Point a->partials / a->counters at the fixed array (set up on first use on
// this device) after checking the request fits it.  The caller has validated
// everything else about the request.
int attn_fixed_scratch_bind(mie_attn_args* a, cudaStream_t st) {
  if (a->num_heads <= 0 || a->splits <= 0) return MIE_ERR_INVALID;
  if (a->num_heads > kFixedCounters ||
      (int64_t)a->num_heads * a->splits * (a->head_dim + 2) > kFixedPartialFloats)
    return MIE_ERR_SCRATCH_LIMIT;
  void* base = nullptr;
  const int rc = fixed_scratch_setup(&base, st);
  if (rc) return rc;
  a->counters = static_cast<uint32_t*>(base);
  a->partials = reinterpret_cast<float*>(static_cast<uint32_t*>(base) + kFixedCounters);
  a->max_splits = a->splits;  // partials packed as [heads, splits, head_dim + 2]
  return MIE_OK;
}

}  // namespace mie
