// Single-query (decode) attention over a paged or contiguous K/V cache, sm_100a.
//
// Reference: src/moe_engine/paged_attention.py:47-154 (one Triton program per
// head looping over 128-token tiles with an online softmax) and the contiguous
// SDPA decode at src/moe_engine/model.py:261-266.
//
// Here the context of every head is split over `splits` CTAs (grid = splits x
// heads) so all SMs stream K/V.  Rows of whole 16-byte pieces run the
// pipelined kernel further down (bulk copies of whole blocks into a ring of
// stages, one online softmax per warp).  The kernel below keeps the rest (and
// is the layout's fallback): a CTA walks its token range in stages of up
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
// The pipelined kernel (rows of whole 16-byte pieces; the kernel above keeps
// the narrow rows).  256 threads = 8 warps.  The split's token range is cut
// into stages of whole blocks (~32 KB of K + V each) held in a ring of up to
// kFastStages slots.  The split's physical block ids are read into shared
// memory first; then warp 0 issues one bulk copy per block for K and one for
// V (a block's K, and its V, is one contiguous run), each stage counted in
// bytes on the mbarrier of its slot, the whole ring in flight at once.  Every
// warp runs its own online softmax (running max and normaliser, HD/32 output
// dims per lane) over its share of each stage as soon as that stage lands --
// no block barrier per stage -- and the eight warp states are merged once at
// the end.  A slot is refilled by warp 0 once every warp arrived on its empty
// barrier.  Stages holding only old tokens are issued before the
// programmatic-dependent wait.
// ---------------------------------------------------------------------------
constexpr int kFastThreads = 256;
constexpr int kFastWarps = kFastThreads / 32;
constexpr int kFastStages = 8;                   // ring slots (at most)
constexpr uint32_t kFastStageBytes = 32 * 1024;  // K + V of one stage (at least one block)
constexpr uint32_t kFastRingBytes = 96 * 1024;   // two CTAs per SM

// two adjacent elements (4- or 8-byte aligned) as floats
__device__ __forceinline__ float2 load2(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}
__device__ __forceinline__ float2 load2(const float* p) { return *reinterpret_cast<const float2*>(p); }

template <typename KV, int HD>
__global__ void __launch_bounds__(kFastThreads) attn_fast_kernel(const mie_attn_args a, AttnLayout L) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr unsigned kAll = 0xffffffffu;
  constexpr int VPT = 16 / (int)sizeof(KV), VPH = HD / VPT;  // 16-byte pieces per row
  // lanes per token in the score pass (VPH rounded up to a power of two),
  // tokens per pass, output dims per lane
  constexpr int LG = VPH <= 1 ? 1 : VPH <= 2 ? 2 : VPH <= 4 ? 4 : VPH <= 8 ? 8 : VPH <= 16 ? 16 : 32;
  constexpr int TPP = 32 / LG;
  constexpr int DPL = (HD + 31) / 32;
  constexpr int P = 4;  // passes per iteration (16 tokens of a warp at hd 64 bf16: one 32 KB stage)
  constexpr uint32_t kRow = HD * sizeof(KV);
  const int h = blockIdx.y, s = blockIdx.x, S = gridDim.x, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int bs = a.block_size, stok = L.chunk_tok, NS = L.nstage;
  int* blk_s = reinterpret_cast<int*>(smem + L.off_blk);
  KV* ring = reinterpret_cast<KV*>(smem + L.off_kv);       // [NS][K | V][stok][HD]
  float* pw = reinterpret_cast<float*>(smem + L.off_acc);  // [warps][HD + 2]: acc, m, l
  __shared__ int last_s;
  __shared__ __align__(8) uint64_t full_s[kFastStages], empty_s[kFastStages];

  // context length (see the kernel above: the device position may be read
  // before the dependency wait; out-of-range values are clamped, reported later)
  int ctx = a.ctx_dev ? (__ldcg(a.ctx_dev) + a.ctx_dev_offset) : a.ctx_len;
  const bool bad_ctx = ctx < 1 || ctx > a.max_ctx;
  if (bad_ctx) ctx = ctx < 1 ? 1 : a.max_ctx;
  const int nblk = (ctx + bs - 1) / bs;
  int b0, b1;
  split_range(nblk, s, S, &b0, &b1);
  const int tok0 = b0 * bs, tok1 = min(b1 * bs, ctx), ntok = max(0, tok1 - tok0);
  const int nst = (ntok + stok - 1) / stok;
  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full_s[i], 1u);
      mbar_init(&empty_s[i], (uint32_t)kFastWarps);
    }
    fence_barrier_init();
  }
  for (int i = tid; i < b1 - b0 && i < L.cap_blocks; i += kFastThreads) {
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
  // Stage i -> slot i % NS (warp 0).  Lane 0 arms the slot's barrier with the
  // stage's bytes, then one lane per block issues its K and V copies (16-byte
  // aligned runs of whole rows: checked on the host).  Stages start on block
  // boundaries (stok is a multiple of bs).
  const int blk_per_stage = stok / bs;
  auto issue = [&](int i) {
    const int t0 = tok0 + i * stok, n = min(stok, tok1 - t0);
    KV* kd = ring + (size_t)(i % NS) * 2 * stok * HD;
    KV* vd = kd + (size_t)stok * HD;
    const int nb = (n + bs - 1) / bs;
    if (lane == 0) {
      fence_proxy_async_smem();  // the slot's earlier reads (ordered by its empty barrier) before the copies
      mbar_arrive_expect_tx(&full_s[i % NS], 2u * (uint32_t)n * kRow);
    }
    __syncwarp();
#pragma unroll 1
    for (int ib = lane; ib < nb; ib += 32) {
      const int64_t blk = blk_s[min(i * blk_per_stage + ib, L.cap_blocks - 1)];
      const uint32_t bytes = (uint32_t)min(bs, n - ib * bs) * kRow;
      const int64_t base = blk * a.stride_block + (int64_t)h * a.stride_head;
      bulk_g2s(kd + (size_t)ib * bs * HD, static_cast<const KV*>(a.k) + base, bytes, &full_s[i % NS]);
      bulk_g2s(vd + (size_t)ib * bs * HD, static_cast<const KV*>(a.v) + base, bytes, &full_s[i % NS]);
    }
  };
  auto landed = [&](int i) { return mbar_wait(&full_s[i % NS], (uint32_t)((i / NS) & 1), a.status); };
  // the split's last stage holds the newest token when the producer grid
  // writes it: issued only after the wait.  `issued` is CTA-uniform until the
  // stage loop, then kept by warp 0 alone.
  const int nst_pre = (a.new_token_last && b1 == nblk && nst > 0) ? nst - 1 : nst;
  int issued = 0;
  for (; issued < min(NS, nst_pre); ++issued)
    if (warp == 0) issue(issued);
  // every issued stage has landed before the CTA leaves (bounded waits)
  auto drain = [&]() {
    for (int i = max(0, issued - NS); i < issued; ++i) landed(i);
  };

  pdl_wait();
  if (skip_requested(a.skip)) {
    drain();
    pdl_trigger();
    return;
  }
  pdl_trigger();
  if (bad_ctx && tid == 0 && s == 0) set_status(a.status, MIE_ERR_RANGE);
  for (; issued < min(NS, nst); ++issued)
    if (warp == 0) issue(issued);

  // this lane's piece of q (score pass: LG lanes per token, lane pc holds
  // elements [pc * VPT, pc * VPT + VPT) of the row)
  const int pc = lane % LG, grp = lane / LG;
  const bool has_piece = pc < VPH;
  float qr[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) qr[j] = has_piece ? load_any(a.q, a.q_dtype, (int64_t)h * HD + pc * VPT + j) : 0.f;
  const float scale = a.scale;
  float m = -INFINITY, l = 0.f, acc[DPL];
#pragma unroll
  for (int d = 0; d < DPL; ++d) acc[d] = 0.f;
  bool lost = false;  // a wait of this warp ran out (status set)
#pragma unroll 1
  for (int i = 0; i < nst; ++i) {
    if (!__all_sync(kAll, landed(i))) {
      lost = true;
      break;
    }
    const int n = min(stok, tok1 - (tok0 + i * stok));
    const KV* kst = ring + (size_t)(i % NS) * 2 * stok * HD;
    const KV* vst = kst + (size_t)stok * HD;
    // this warp's tokens [wa, wb) of the stage, TPP per pass
    const int wa = n * warp / kFastWarps, wb = n * (warp + 1) / kFastWarps;
    // P passes of TPP tokens per iteration: their dot products, shuffle
    // reductions and exps are independent chains, one max / sum reduction
    // and one rescale for all of them
#pragma unroll 1
    for (int t = wa; t < wb; t += P * TPP) {
      float sv[P];
#pragma unroll
      for (int u = 0; u < P; ++u) {
        const int tt = t + u * TPP + grp;
        sv[u] = (tt < wb && has_piece)
                    ? dot_vec(reinterpret_cast<const uint4*>(kst + (size_t)tt * HD)[pc], qr, 0.f, (const KV*)nullptr)
                    : 0.f;
      }
#pragma unroll
      for (int o = 1; o < LG; o <<= 1)
#pragma unroll
        for (int u = 0; u < P; ++u) sv[u] += __shfl_xor_sync(kAll, sv[u], o);
      float mx = -INFINITY;
#pragma unroll
      for (int u = 0; u < P; ++u) {
        sv[u] = (t + u * TPP + grp < wb) ? sv[u] * scale : -INFINITY;
        mx = fmaxf(mx, sv[u]);
      }
#pragma unroll
      for (int o = LG; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(kAll, mx, o));
      const float mn = fmaxf(m, mx);  // finite: token t is live
      const float alpha = expf(m - mn);
      float pr[P], ps = 0.f;
#pragma unroll
      for (int u = 0; u < P; ++u) {
        pr[u] = sv[u] == -INFINITY ? 0.f : expf(sv[u] - mn);
        ps += pr[u];
      }
#pragma unroll
      for (int o = LG; o < 32; o <<= 1) ps += __shfl_xor_sync(kAll, ps, o);
      l = fmaf(l, alpha, ps);
      m = mn;
      float ac[2][DPL];
#pragma unroll
      for (int d = 0; d < DPL; ++d) {
        ac[0][d] = acc[d] * alpha;
        ac[1][d] = 0.f;
      }
#pragma unroll
      for (int u = 0; u < P; ++u) {
#pragma unroll
        for (int k = 0; k < TPP; ++k) {
          const float pk = __shfl_sync(kAll, pr[u], k * LG);
          const int tk = t + u * TPP + k;
          float* av = ac[(u * TPP + k) & 1];
          if (tk < wb) {
            const KV* vr = vst + (size_t)tk * HD;
            if constexpr (DPL == 2 && HD == 64) {
              const float2 v2 = load2(vr + 2 * lane);
              av[0] = fmaf(pk, v2.x, av[0]);
              av[1] = fmaf(pk, v2.y, av[1]);
            } else {
#pragma unroll
              for (int d = 0; d < DPL; ++d) {
                const int dd = lane * DPL + d;
                if (dd < HD) av[d] = fmaf(pk, Elem<KV>::to_f(vr[dd]), av[d]);
              }
            }
          }
        }
      }
#pragma unroll
      for (int d = 0; d < DPL; ++d) acc[d] = ac[0][d] + ac[1][d];
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_s[i % NS]);  // this warp no longer reads the slot
    if (warp == 0 && issued < nst) {
      // refill slot i % NS with stage issued == i + NS once every warp left it
      if (!__all_sync(kAll, mbar_wait(&empty_s[i % NS], (uint32_t)((i / NS) & 1), a.status))) {
        lost = true;
        break;
      }
      issue(issued);
      ++issued;
    }
  }

  // ---- merge the warps: (acc, m, l) of every warp -> the CTA's partial ----
#pragma unroll
  for (int d = 0; d < DPL; ++d) {
    const int dd = lane * DPL + d;
    if (dd < HD) pw[warp * (HD + 2) + dd] = acc[d];
  }
  if (lane == 0) {
    pw[warp * (HD + 2) + HD] = m;
    pw[warp * (HD + 2) + HD + 1] = l;
  }
  if (__syncthreads_or(lost) && warp == 0) drain();
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < kFastWarps; ++w) M = fmaxf(M, pw[w * (HD + 2) + HD]);
  float lsum = 0.f, o = 0.f;
#pragma unroll
  for (int w = 0; w < kFastWarps; ++w) {
    const float mw = pw[w * (HD + 2) + HD];
    if (mw != -INFINITY) {
      const float e = expf(mw - M);
      lsum = fmaf(e, pw[w * (HD + 2) + HD + 1], lsum);
      if (tid < HD) o = fmaf(e, pw[w * (HD + 2) + tid], o);
    }
  }
  const bool direct_out = (S == 1 && !a.defer_merge);
  float* part = a.partials + ((size_t)h * a.max_splits + s) * (HD + 2);
  if (tid < HD) {
    if (direct_out)
      store_any(a.out, a.out_dtype, (int64_t)h * HD + tid, lsum > 0.f ? o / lsum : 0.f);
    else
      part[2 + tid] = o;
  }
  if (direct_out) return;
  if (tid == 0) {
    part[0] = M;
    part[1] = lsum;
  }
  if (a.defer_merge) return;
  // arrival: the block barrier orders every thread's partial stores before
  // thread 0's release (gpu scope) on the head's counter; the last arrival's
  // acquire, then the barrier, orders the other splits' partials before this
  // CTA's loads
  __syncthreads();
  if (tid == 0) last_s = (atom_add_acq_rel_gpu(a.counters + h, 1u) == (uint32_t)(S - 1));
  __syncthreads();
  if (!last_s) return;
  // log-sum-exp merge of the S partials of this head, staged in shared memory
  // (the ring is free) with every thread's loads in flight together
  const float* hp = a.partials + (size_t)h * a.max_splits * (HD + 2);
  float* ps = reinterpret_cast<float*>(ring);  // [S][HD + 2]
  const int np = S * (HD + 2);
  constexpr int T = kFastThreads;
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
  // per-split weights e^(m_j - M) and the normaliser once (warp 0), then
  // Q subsets of the splits per output dim, summed at the end
  float* wts = ps + np;  // [S]
  float* osum = wts + S;  // [Q][HD]
  __shared__ float lsum_s;
  if (warp == 0) {
    float mloc = -INFINITY;
    for (int j = lane; j < S; j += 32) mloc = fmaxf(mloc, ps[j * (HD + 2)]);
    const float Mh = warp_max(mloc);
    float lw = 0.f;
    for (int j = lane; j < S; j += 32) {
      const float mj = ps[j * (HD + 2)];
      const float w = mj == -INFINITY ? 0.f : expf(mj - Mh);
      wts[j] = w;
      lw = fmaf(w, ps[j * (HD + 2) + 1], lw);
    }
    lw = warp_sum(lw);
    if (lane == 0) lsum_s = lw;
  }
  __syncthreads();
  constexpr int Q = T / HD;
  if (tid < Q * HD) {
    const int d = tid % HD, qq = tid / HD;
    float o2 = 0.f;
    for (int j = qq; j < S; j += Q) o2 = fmaf(wts[j], ps[j * (HD + 2) + 2 + d], o2);
    osum[qq * HD + d] = o2;
  }
  __syncthreads();
  for (int d = tid; d < HD; d += T) {
    float o2 = 0.f;
#pragma unroll
    for (int qq = 0; qq < Q; ++qq) o2 += osum[qq * HD + d];
    store_any(a.out, a.out_dtype, (int64_t)h * HD + d, o2 / lsum_s);
  }
  if (tid == 0) a.counters[h] = 0u;  // ready for the next launch
}

// The pipelined kernel exists for rows of whole 16-byte pieces only.
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
  // 16-byte rows run the pipelined kernel: a ring of stages of whole blocks
  // (~32 KB of K + V each, up to 96 KB), the split's block ids, per-warp
  // partial states
  if ((a.head_dim * esz) % 16 == 0 && a.splits > 0) {
    AttnLayout F{};
    F.fast = 1;
    int ct = (int)(kFastStageBytes / (uint32_t)per_tok) / a.block_size * a.block_size;
    if (ct < a.block_size) ct = a.block_size;
    F.chunk_tok = ct;
    int ns = (int)(kFastRingBytes / ((uint32_t)per_tok * (uint32_t)ct));
    F.nstage = ns < 1 ? 1 : (ns > kFastStages ? kFastStages : ns);
    const int max_blk = (a.max_ctx + a.block_size - 1) / a.block_size;
    F.cap_blocks = (max_blk + a.splits - 1) / a.splits;
    if (F.cap_blocks < 1) F.cap_blocks = 1;
    off = 0;
    F.off_kv = take((size_t)F.nstage * per_tok * ct);
    F.off_blk = take(sizeof(int) * (size_t)F.cap_blocks);
    F.off_acc = take(sizeof(float) * kFastWarps * (size_t)(a.head_dim + 2));
    F.smem = (uint32_t)((off + 127) & ~size_t(127));
    // the merge stages every split's partial, its weight and the dim sums in the ring
    if (((size_t)a.splits * (a.head_dim + 3) + kFastThreads) * 4 <= (size_t)F.nstage * per_tok * ct &&
        F.smem <= (uint32_t)kMaxDynSmem)
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
