// Persistent decode step on thread-block clusters, sm_100a.
//
// The whole batch-one decode step (all layers + LM head) in ONE launch, like
// the one-CTA-per-SM step of step.cu, but laid out on clusters of
// kStepCluster (6) CTAs so that the work that stays inside one attention head
// synchronises through distributed shared memory (a cluster barrier, ~0.25 us
// on B200) instead of device-wide exchanges (~1.1 us each), and so that no
// CTA repeats another's work.  Shapes: bf16 weights and cache, head_dim 64,
// hidden <= 768, RMSNorm, RoPE, SwiGLU experts, top-2, no biases, greedy
// argmax -- the BASELINE miniMoE family; the dataflow is the reference's
// decode step (src/moe_engine/model.py:494-498, 543-565).
//
// Grid: NC clusters (as many as the GPU holds at once: 22 on a 148-SM B200,
// 132 CTAs), 512 threads per CTA.  Cluster h < num_heads is head h's
// attention group; CTA s of it is split s of the head's old tokens and owns
// RoPE pairs / v rows / out_proj rows share s of the head.
//
// Per layer l (tags (step << 8) | l on every exchange word):
//
//   ATT (attention clusters)
//     x <- exchange X (or the token embedding at l = 0); RMSNorm
//     this CTA's q and k rows (whole RoPE pairs) and v rows from shared
//       memory; RoPE; k, v rounded to the cache type and stored into the
//       position's cache slot; q, k_new, v_new sent to every CTA of the
//       cluster (DSMEM) -- cluster barrier 1
//     online softmax over this split's old tokens (staged K/V chunk)
//     (m, l, acc) sent to every CTA of the cluster -- cluster barrier 2
//     every CTA merges the head (log-sum-exp, the new token as one more
//       term) -> o_h [hd]; its out_proj rows times o_h (a TMA tile of
//       out_proj's columns of head h) -> exchange P[h] (the head's partial
//       of out_proj . o)
//   MOE (every cluster)
//     CTA s receives rows share s of P (every head) and of x, sums them
//       (x_mid = x + sum_h P[h]) and sends its rows, their square sum and
//       their router partial dots (x_mid * norm w) . router row e to every
//       CTA of the cluster -- cluster barrier 3
//     routing from the cluster's shares: RMSNorm scale, logits, top-2 (ties
//       to the lower id), 2-way softmax -- computed by every consumer warp
//       and by the producer warp, which bulk-copies the selected experts'
//       gate/up rows of this CTA's units and down rows of its output rows
//       into shared memory while the consumers normalise x_mid
//     up units: silu(gate) * up -> exchange H
//     down rows of both slots . h + residual -> exchange X of layer l + 1
//
// The RMSNorms before the q/k/v rows and the LM head are folded into the
// receive of x: the GEMVs run on x * w and their results are scaled by rs.
//
// HEAD: x_L -> final norm -> this CTA's tied LM-head rows (a ring of bulk
// copies) -> argmax -> the last CTA reduces the CTA results and does the
// step's device bookkeeping (token, position + 1, token log, EOS flag).
//
// Weights never pass through registers ahead of use: every GEMV reads rows
// that bulk copies (cp.async.bulk / cp.async.bulk.tensor, no multicast) put
// in shared memory earlier -- the next layer's q/k/v rows right after this
// layer's up GEMV, its K/V chunk right after this layer's attention, its
// out_proj tile right after this layer's out_proj, its router and norm
// weights right after this layer's routing.
//
// Buffer reuse.  Device-wide exchange buffers alternate by layer parity; a
// copy is rewritten two layers later only after every CTA consumed it (the
// data dependencies of the layer in between order the reads first).  The
// cluster gather buffers alternate by layer parity as well, and every remote
// write happens just before a cluster barrier that every CTA of the cluster
// passes after its last read of the previous use.
//
// Failure.  Every wait is bounded (mie_step_desc.wait_limit_ns).  A CTA that
// gives up records MIE_ERR_TIMEOUT and raises the abort word; from then on it
// runs the step's program without waiting, computing or writing -- but it
// still takes every cluster barrier, so no CTA of its cluster is ever left
// waiting at one -- drains its bulk copies and leaves.  The host zeroes the
// scratch before the next step.
//
// Every reduction has a fixed order: results are bit-reproducible, and every
// CTA that computes a value redundantly (x_mid, the router's choice, o_h)
// computes the same bits.
#include <mutex>

#include "exchange.cuh"
#include "kernels.h"
#include "stream.cuh"

namespace mie {

namespace {

using bf16 = __nv_bfloat16;
constexpr int kT = kStepThreads;      // 512 threads
constexpr int kW = kT / 32;           // 16 warps
constexpr int kCT = kT - 32;          // consumer threads: warps 0..14
constexpr int kCW = kCT / 32;         // consumer warps
constexpr int kProd = kCT;            // first thread of the producer warp (warp 15)
constexpr int kCS = kStepCluster;     // CTAs per cluster
constexpr int kHd = kClusterHeadDim;  // head_dim
constexpr int kPV = 8;                // bf16 elements per 16-byte vector
constexpr int kMg = kHd + 4;          // merge partial: acc [hd], m, l (padded)

constexpr int kHdrStep = 0, kHdrAbort = 1;  // scratch header words

// "Full" mbarriers (a staged region landed), each filled by one side:
// the producer warp (count 1: lane 0 arrives with the bytes expected) --
// q/k/v rows (region A), the first K/V chunk (K), the out_proj tile (O),
// router + norm weights (R), the selected experts' gate/up rows (A) and down
// rows (D), the LM-head ring stages -- or the consumers (count kCT) --
// further K/V chunks (K).  "Empty" mbarriers (count 1,
// arrived by consumer thread 0): a region the producer refills was read for
// the last time.
constexpr int kFQ = 0, kFK = 1, kFK2 = 2, kFO = 3, kFR = 4, kFE = 5, kFD = 6, kFH = 7;
constexpr int kNF = kFH + kStepHeadStagesMax;  // full barriers
constexpr int kEK = kNF, kEO = kNF + 1, kER = kNF + 2, kEA = kNF + 3, kED = kNF + 4, kEH = kNF + 5;
constexpr int kNB = kEH + kStepHeadStagesMax;
constexpr int kBlkCache = 64;  // block ids of a split cached per step

#ifdef MIE_STEP_STAMPS
constexpr int kStampLayers = kMaxStepLayers + 1, kStampPoints = 32;
__device__ unsigned long long g_cstep_stamps[160 * kStampLayers * kStampPoints];
// SM cycle counter (clock64): durations inside one CTA are exact
#define CSTAMP(l, k)                                                                                   \
  do {                                                                                                 \
    if (threadIdx.x == 0) g_cstep_stamps[(blockIdx.x * kStampLayers + (l)) * kStampPoints + (k)] = clock64(); \
  } while (0)
#else
#define CSTAMP(l, k) \
  do {               \
  } while (0)
#endif

struct CCtx {
  int pos;        // position of the input token
  int stop;       // nonzero: skip the step (EOS reached, step limit, bad input)
  uint32_t step;  // this step's number (tags)
  int64_t tok;    // input token
  int64_t slot;   // cache offset of the new token's slot (head 0)
  int last;       // this CTA finished the LM head last
  int blk0;       // first cache block of this CTA's old tokens
  int log_k;      // *log_count at the start of the step
  int sel0, sel1; // the layer's experts
  float wt0, wt1; // and their weights
  float snew;     // scale * q . k_new
  uint32_t pstep; // expert parallel: the group's step number (tags of the cross-GPU exchange)
};
__shared__ CCtx cx;
__shared__ unsigned long long lim_s;  // limit of every wait (ns)
struct CShared {
  mie_step_desc d;
  CGeom g;
};
__shared__ CShared ps;
constexpr int kLaySlots = 4;
__shared__ mie_layer_desc lay_s[kLaySlots];
__shared__ float red_s[kW], red2_s[kW];
__shared__ int blk_s[kBlkCache];
__shared__ float bestv_s[kW];
__shared__ int besti_s[kW];
__shared__ __align__(8) uint64_t bars_s[kNB];
__shared__ uint32_t armed_s[kNB], done_s[kNB];
__shared__ uint32_t wdone_s[kCW][kNF];  // full-barrier phases each consumer warp has waited for
extern __shared__ __align__(128) uint8_t sm[];

template <typename T>
__device__ __forceinline__ T* at(uint32_t off) {
  return reinterpret_cast<T*>(sm + off);
}
__device__ __forceinline__ const mie_layer_desc& layer_at(int l) { return lay_s[l & (kLaySlots - 1)]; }
__device__ __forceinline__ uint32_t tag_of(int l) { return (cx.step << 8) | (uint32_t)l; }
// Tags of the cross-GPU exchange (expert parallel): the top bit keeps them
// apart from the per-layer MoE kernels' call numbers in the same buffers.
__device__ __forceinline__ uint32_t ptag_of(int l) {
  return 0x80000000u | ((cx.pstep & 0x7fffffu) << 8) | (uint32_t)l;
}
__device__ __forceinline__ void split32(int total, int c, int g, int* b, int* e) {
  *b = (int)(((uint32_t)total * (uint32_t)c) / (uint32_t)g);
  *e = (int)(((uint32_t)total * (uint32_t)(c + 1)) / (uint32_t)g);
}
__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }
__device__ __forceinline__ void raise_abort() {
  atomicExch(reinterpret_cast<unsigned long long*>(ps.g.ll + kHdrAbort), 1ull);
}
// Barrier over the consumer warps (named barrier 1); the producer warp never
// takes it.
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kCT) : "memory"); }
__device__ __forceinline__ int csync_or(int v) {
  uint32_t any;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbarrier.red.or.pred p, 1, %2, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(any)
      : "r"(v), "n"(kCT)
      : "memory");
  return (int)any;
}
__device__ __forceinline__ void mbar_arrive1(int b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&bars_s[b])) : "memory");
}
// Consumer thread 0, after the consumer barrier that follows the last read of
// a region: tell the producer the region is free.
__device__ __forceinline__ void region_free(int b) {
  if (threadIdx.x == 0) mbar_arrive1(b);
}
// Cluster barrier in two halves (the producer warp arrives early and waits
// late, so the consumers never wait for it).
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
__device__ __forceinline__ void layer_fetch(const CStepParams& P, int l, int first) {
  constexpr int kWords = (int)(sizeof(mie_layer_desc) / 8);
  const int i = (int)threadIdx.x - first;
  if (i >= 0 && i < kWords)
    reinterpret_cast<uint64_t*>(&lay_s[l & (kLaySlots - 1)])[i] = reinterpret_cast<const uint64_t*>(&P.layers[l])[i];
}

// ---------------------------------------------------------------------------
// Bounded waits.  Each returns a CTA-uniform result: true when `ok` was
// true and every thread's wait succeeded; a CTA that is no longer ok skips
// the wait (but still takes the block barrier).
// ---------------------------------------------------------------------------
// Slow path of a poll, every 64 rounds: true when another CTA raised the
// abort word or this wait ran out (then MIE_ERR_TIMEOUT, abort raised).
__device__ __noinline__ bool give_up(unsigned long long* t0) {
  if (ll_ld(ps.g.ll + kHdrAbort)) return true;
  const unsigned long long t = global_ns();
  if (!*t0) {
    *t0 = t;
    return false;
  }
  if (t - *t0 <= lim_s) return false;
  set_status(ps.d.status, MIE_ERR_TIMEOUT);
  raise_abort();
  return true;
}

// Poll n exchange words: dst[i] = value of buf[src(i)] once its tag equals
// `tag`.  Consumer thread t owns words t, t + kCT, ... in groups of four
// polled together.  1 when this thread gave up.
template <typename Src>
__device__ __forceinline__ int poll(const uint64_t* buf, int n, uint32_t tag, float* dst, Src src) {
  unsigned long long t0 = 0;
#pragma unroll 1
  for (int i0 = threadIdx.x; i0 < n; i0 += 4 * kCT) {
    uint64_t w[4];
    int a[4];
    unsigned need = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = i0 + j * kCT;
      a[j] = i < n ? src(i) : 0;
      if (i < n) {
        w[j] = ll_ld(buf + a[j]);
        need |= 1u << j;
      }
    }
#pragma unroll 1
    for (int it = 1;; ++it) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if ((need >> j & 1u) && ll_tag(w[j]) == tag) {
          dst[i0 + j * kCT] = ll_val(w[j]);
          need &= ~(1u << j);
        }
      if (!need) break;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (need >> j & 1u) w[j] = ll_ld(buf + a[j]);
      if ((it & 63) == 0 && give_up(&t0)) return 1;
    }
  }
  return 0;
}
struct Ident {
  __device__ __forceinline__ int operator()(int i) const { return i; }
};

// ---------------------------------------------------------------------------
// Expert parallel: exchange X across GPUs.  Every rank's down-row owners store
// their rows of the rank's MoE partial (the contribution of the selected
// experts it holds, 0 for the others) into slot [layer parity][rank] of every
// rank's buffer; a reader sums the ranks' words of a row in rank order and
// adds x_mid -- the combine of the per-layer expert-parallel path, so every
// rank computes the same bits of x (and the same routing).
//
// Slot reuse: the layer outputs of all steps form one sequence (index
// seq * L + l, seq the group's step counter before the step) and alternate
// between the two slots along it, across step boundaries too.  Every rank
// writes every row of every layer output, and a rank writes output n + 2 only
// after it read output n + 1 completely -- whose words every other rank wrote
// after all its CTAs had read output n (it needed their expert units).  So a
// slot is rewritten only after every rank read it.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t pslot(int l) {
  return ((cx.pstep - 1u) * (uint32_t)ps.d.num_layers + (uint32_t)l) & 1u;
}
__device__ __forceinline__ void peer_put(int l, int r, float y) {
  const CGeom& g = ps.g;
  const size_t o = ((size_t)pslot(l) * g.peer_world + g.peer_rank) * ps.d.hidden_dim + r;
  const uint32_t t = ptag_of(l);
#pragma unroll 1
  for (int k = 0; k < g.peer_world; ++k) ll_put_sys(g.peer_bufs[k] + o, y, t);
}

// Rows a0 + i, i < n, of layer l's X from this GPU's buffer: dst[i] =
// base[a0 + i] + (sum over ranks in rank order of the rank's word).  dst may
// be base.  1 when this thread gave up.
__device__ __noinline__ int poll_ranks(int l, int n, const float* base, float* dst, int a0) {
  const CGeom& g = ps.g;
  const int D = ps.d.hidden_dim, W = g.peer_world;
  const uint64_t* buf = g.peer_bufs[g.peer_rank] + (size_t)pslot(l) * W * D;
  const uint32_t tag = ptag_of(l);
  unsigned long long t0 = 0;
#pragma unroll 1
  for (int i = threadIdx.x; i < n; i += kCT) {
    const int a = a0 + i;
    uint64_t w[MIE_PEER_MAX_RANKS];
    unsigned need = 0;
#pragma unroll
    for (int k = 0; k < MIE_PEER_MAX_RANKS; ++k)
      if (k < W) {
        w[k] = ll_ld_sys(buf + (size_t)k * D + a);
        need |= 1u << k;
      }
#pragma unroll 1
    for (int it = 1;; ++it) {
#pragma unroll
      for (int k = 0; k < MIE_PEER_MAX_RANKS; ++k)
        if ((need >> k & 1u) && ll_tag(w[k]) == tag) need &= ~(1u << k);
      if (!need) break;
#pragma unroll
      for (int k = 0; k < MIE_PEER_MAX_RANKS; ++k)
        if (need >> k & 1u) w[k] = ll_ld_sys(buf + (size_t)k * D + a);
      if ((it & 63) == 0 && give_up(&t0)) return 1;
    }
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < MIE_PEER_MAX_RANKS; ++k)
      if (k < W) s += ll_val(w[k]);
    dst[i] = base[a] + s;
  }
  return 0;
}

// A consumer warp: wait (bounded) for the next phase of full barrier b.
// Every thread observes the phase itself (which also makes the staged bytes
// visible to it), so no barrier is needed; the result is warp-uniform and
// becomes CTA-uniform at the next consumer barrier that carries it.
__device__ __noinline__ bool bwait(bool ok, int b) {
  if (!ok) return false;
  const int w = threadIdx.x >> 5;
  const uint32_t k = wdone_s[w][b];
  const bool mine = mbar_wait(&bars_s[b], k & 1u, ps.d.status, lim_s);
  if (!mine) raise_abort();
  const bool all = __all_sync(0xffffffffu, mine);
  __syncwarp();
  if (all && (threadIdx.x & 31) == 0) wdone_s[w][b] = k + 1;
  __syncwarp();
  return all;
}

// Producer warp: wait (bounded) for the next phase of empty barrier b.
__device__ __noinline__ bool pwait(bool ok, int b) {
  if (!ok) return false;
  const bool mine = mbar_wait(&bars_s[b], done_s[b] & 1u, ps.d.status, lim_s);
  if (!mine) raise_abort();
  const bool all = __all_sync(0xffffffffu, mine);
  __syncwarp();
  if (all && (threadIdx.x & 31) == 0) done_s[b] += 1;
  __syncwarp();
  return all;
}

// Before leaving: wait (bounded) for every armed copy not waited for, so no
// copy lands in shared memory after the CTA left.
__device__ __noinline__ void drain_copies() {
  __syncthreads();
  if (threadIdx.x != 0) return;
#pragma unroll 1
  for (int b = 0; b < kNF; ++b) {
    uint32_t k = wdone_s[0][b];  // phases consumer warp 0 waited for
    while (k < armed_s[b]) {
      mbar_wait(&bars_s[b], k & 1u, nullptr);
      ++k;
    }
  }
}

// ---------------------------------------------------------------------------
// Consumer staging: right after routing the consumer warps, which would
// otherwise only wait, fill the expert regions themselves with 16-byte
// cp.async copies (chunk j by consumer thread j mod kCT); every consumer
// thread then arrives on the region's full barrier once its own copies landed
// (cp.async.mbarrier.arrive.noinc).  Spread over 15 warps, the issue keeps
// enough bytes in flight; the same copies from one warp would not.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp16(void* dst, const void* src, uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "l"(pol)
               : "memory");
}
// Staging side of the calling thread: (index, count).
struct Side {
  int i, n;
};
__device__ __forceinline__ Side cons_side() { return Side{(int)threadIdx.x, kCT}; }
// After this side's copies of one phase of full barrier b: arrive when they land.
__device__ __forceinline__ void stage_done(Side sd, int b) {
  if (sd.i == 0) armed_s[b] += 1;
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(&bars_s[b])) : "memory");
}

struct Split {
  int h, s;        // head (cluster), split (rank)
  int p0, np;      // RoPE pairs [p0, p0 + np)
  int v0, nv;      // v rows
  int t0, t1;      // old tokens
  int r0, nr;      // out_proj rows
};
__device__ __forceinline__ Split split_of(int pos) {
  Split a;
  a.h = blockIdx.x / kCS;
  a.s = blockIdx.x % kCS;
  int e;
  split32(kHd / 2, a.s, kCS, &a.p0, &e);
  a.np = e - a.p0;
  split32(kHd, a.s, kCS, &a.v0, &e);
  a.nv = e - a.v0;
  split32(pos, a.s, kCS, &a.t0, &a.t1);
  split32(ps.d.hidden_dim, a.s, kCS, &a.r0, &e);
  a.nr = e - a.r0;
  return a;
}

// K/V of tokens [ta, ta + n) of head h, layer l -> region K (K rows, then V
// rows at chunk_tok): 16-byte piece j of the n K rows then of the n V rows,
// each through the block table.
__device__ __noinline__ void issue_kv(Side sd, int b, int l, int h, int ta, int n) {
  const mie_step_desc& d = ps.d;
  const mie_layer_desc& ly = layer_at(l);
  const int bs = d.block_size;
  constexpr int kPieces = kHd / kPV;
  bf16* dst = at<bf16>(ps.g.sm_k);
  const uint64_t pol = policy_evict_first();
  const int total = 2 * n * kPieces;
#pragma unroll 1
  for (int j = sd.i; j < total; j += sd.n) {
    const int v = j >= n * kPieces;
    const int jj = j - v * n * kPieces, t = jj / kPieces, q = jj - t * kPieces;
    const int tok = ta + t, bi = tok / bs;
    int64_t blk = bi;
    if (d.block_table) {
      const int k = bi - cx.blk0;
      const int pb = (k >= 0 && k < kBlkCache) ? blk_s[k] : __ldg(d.block_table + bi);
      if (pb < 0 || pb >= d.num_blocks) set_status(d.status, MIE_ERR_RANGE);
      blk = (pb < 0 || pb >= d.num_blocks) ? 0 : pb;
    }
    const int64_t off =
        blk * d.kv_stride_block + (int64_t)h * d.kv_stride_head + (int64_t)(tok % bs) * d.kv_stride_tok + q * kPV;
    cp16(dst + (size_t)v * ps.g.chunk_tok * kHd + (size_t)t * kHd + q * kPV,
         static_cast<const bf16*>(v ? ly.v_cache : ly.k_cache) + off, pol);
  }
  stage_done(sd, b);
}

// ---------------------------------------------------------------------------
// Producer staging: bulk (TMA) copies issued by the producer warp, counted in
// bytes on the region's full barrier (armed by one lane with expect_tx).  One
// thread issues a large copy and the copy engine moves the bytes, while a
// warp issuing 16-byte cp.async copies keeps only a few kilobytes in flight.
// Issuing holds the producer warp for 0.1-0.4 us per copy, off the
// consumers' path.  Each copy follows a proxy fence: the consumers read the
// region with ordinary loads before the empty barrier released it.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void bar_arm(int b, uint32_t bytes) {
  armed_s[b] += 1;
  mbar_arrive_expect_tx(&bars_s[b], bytes);
}
__device__ __noinline__ void bulk_copy(void* dst, const void* src, uint32_t bytes, int b, bool keep = false) {
  const uint64_t pol = keep ? policy_evict_last() : policy_evict_first();
#pragma unroll 1
  for (uint32_t o = 0; o < bytes; o += kBulkMax)
    bulk_g2s_stream(static_cast<uint8_t*>(dst) + o, static_cast<const uint8_t*>(src) + o, min(kBulkMax, bytes - o),
                    &bars_s[b], pol);
}

// Layer l's q/k/v rows of this split -> region A (producer warp: lane 0 arms,
// lanes 0-4 issue one copy each: q pair first halves, second halves, k pair
// first halves, second halves, v rows).
__device__ __noinline__ void tma_qkv(int l) {
  const mie_step_desc& d = ps.d;
  const Split a = split_of(cx.pos);
  const int lane = threadIdx.x & 31, D = d.hidden_dim;
  const uint32_t rb = (uint32_t)D * 2u;
  if (lane == 0) {
    fence_proxy_async_smem();
    bar_arm(kFQ, (uint32_t)(4 * a.np + a.nv) * rb);
  }
  __syncwarp();
  if (lane > 4) return;
  fence_proxy_async_smem();
  const uint8_t* w = static_cast<const uint8_t*>(layer_at(l).qkv_w);
  uint8_t* dst = at<uint8_t>(ps.g.sm_a);
  const int64_t base = (int64_t)a.h * kHd;
  int64_t row;
  int n, slot;
  if (lane < 4) {
    row = (lane >= 2 ? D : 0) + base + (lane & 1) * (kHd / 2) + a.p0;
    n = a.np;
    slot = lane * a.np;
  } else {
    row = 2 * (int64_t)D + base + a.v0;
    n = a.nv;
    slot = 4 * a.np;
  }
  if (n > 0) bulk_copy(dst + (size_t)slot * rb, w + row * rb, (uint32_t)n * rb, kFQ);
}

// Layer l's out_proj tile of this split (rows [r0, r0 + orows), the hd
// columns of head h; row r of the tile at r * hd elements) -> region O: one
// 2-D tensor copy (producer lane 0).
__device__ __noinline__ void tma_otile(const CStepParams& P, int l) {
  if ((threadIdx.x & 31) != 0) return;
  const Split a = split_of(cx.pos);
  fence_proxy_async_smem();
  bar_arm(kFO, (uint32_t)ps.g.orows * kHd * 2u);
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(at<uint8_t>(ps.g.sm_o))),
      "l"(&P.omap[l]), "r"(a.h * kHd), "r"(a.r0), "r"(smem_u32(&bars_s[kFO])), "l"(policy_evict_first())
      : "memory");
}

// Layer l's router rows and both norm weights -> region R, or for l ==
// num_layers the final norm weights (producer lane 0).
__device__ __noinline__ void tma_side(int l) {
  if ((threadIdx.x & 31) != 0) return;
  const mie_step_desc& d = ps.d;
  const uint32_t rb = (uint32_t)d.hidden_dim * 2u;
  uint8_t* dst = at<uint8_t>(ps.g.sm_r);
  fence_proxy_async_smem();
  if (l == d.num_layers) {
    bar_arm(kFR, rb);
    bulk_copy(at<uint8_t>(ps.g.sm_fn), d.final_norm_w, rb, kFR);
    return;
  }
  const mie_layer_desc& ly = layer_at(l);
  bar_arm(kFR, (uint32_t)(d.num_experts + 2) * rb);
  bulk_copy(dst, ly.router_w, (uint32_t)d.num_experts * rb, kFR);
  bulk_copy(dst + (size_t)d.num_experts * rb, ly.attn_norm_w, rb, kFR);
  bulk_copy(dst + (size_t)(d.num_experts + 1) * rb, ly.moe_norm_w, rb, kFR);
}

// The selected experts' rows of this CTA (producer warp): gate rows then up
// rows of its units -> region A (barrier A), or (down) the down rows of its
// output rows, slot 0 then slot 1 -> region D (barrier D); lane 0 issues at
// most four / two bulk copies.  e0, e1: the slots' experts in this rank's
// weight stack; with EP (expert parallel) -1 marks a slot held by another
// rank, which stages nothing (its barrier phase still completes).  With Q8
// (int8 experts) the rows are int8 and the warp also loads their fp32 group
// scales into the region (after the rows, at q_a_scale / q_d_scale); the
// barrier's one arrival follows those stores, so its phase completes once the
// rows landed and the scales are in place.  Regions A and D were last read
// before cluster barrier 3 of this layer, which the caller has passed.
template <bool EP, bool Q8>
__device__ __noinline__ void tma_experts(int l, int e0, int e1, bool down) {
  static_assert(!(EP && Q8), "int8 experts run without expert parallelism in this kernel");
  const int lane = threadIdx.x & 31;
  if (!Q8 && lane != 0) return;
  const mie_step_desc& d = ps.d;
  const CGeom& g = ps.g;
  const mie_layer_desc& ly = layer_at(l);
  const int D = d.hidden_dim, Hx = d.expert_hidden_dim;
  const uint32_t eb = Q8 ? 1u : 2u;  // bytes per weight
  const uint32_t rbD = (uint32_t)D * eb, rbH = (uint32_t)Hx * eb;
  int u0, u1, r0, r1;
  split32(2 * Hx, blockIdx.x, g.G, &u0, &u1);
  split32(D, blockIdx.x, g.G, &r0, &r1);
  const int nu = u1 - u0, nr = r1 - r0;
  const int b = down ? kFD : kFE;
  if (lane == 0) {
    fence_proxy_async_smem();
    uint32_t bytes = 0;
    if (down) {
      bytes = (uint32_t)((!EP || e0 >= 0) + (!EP || e1 >= 0)) * (uint32_t)nr * rbH;
    } else {
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int ua = max(u0, k * Hx), ub = min(u1, (k + 1) * Hx);
        if (ub > ua && (!EP || (k ? e1 : e0) >= 0)) bytes += 2u * (uint32_t)(ub - ua) * rbD;
      }
    }
    if (Q8) {  // the arrival comes after the scales
      armed_s[b] += 1;
      mbar_expect_tx(&bars_s[b], bytes);
    } else {
      bar_arm(b, bytes);
    }
    if (down) {
#pragma unroll 1
      for (int k = 0; k < 2; ++k) {
        const int e = k ? e1 : e0;
        if (!EP || e >= 0)
          bulk_copy(at<uint8_t>(g.sm_d) + (size_t)k * nr * rbH,
                    static_cast<const uint8_t*>(ly.w2) + ((size_t)e * D + r0) * rbH, (uint32_t)nr * rbH, kFD);
      }
    } else {
#pragma unroll 1
      for (int m = 0; m < 2; ++m) {
        const uint8_t* w = static_cast<const uint8_t*>(m ? ly.w3 : ly.w1);
#pragma unroll 1
        for (int k = 0; k < 2; ++k) {
          const int ua = max(u0, k * Hx), ub = min(u1, (k + 1) * Hx), e = k ? e1 : e0;
          if (ub > ua && (!EP || e >= 0))
            bulk_copy(at<uint8_t>(g.sm_a) + (size_t)(m * nu + ua - u0) * rbD,
                      w + ((size_t)e * Hx + ua - k * Hx) * rbD, (uint32_t)(ub - ua) * rbD, kFE);
        }
      }
    }
  }
  if constexpr (Q8) {
    // the scales in batches of eight independent loads per lane
    constexpr int kB = 8;
    if (down) {
      // scales of the down rows: [slot k][row i][group c]
      const int ng = Hx >> g.qgsh, cnt = 2 * nr * ng;
      float* dst = at<float>(g.sm_d + g.q_d_scale);
#pragma unroll 1
      for (int i0 = lane; i0 < cnt; i0 += 32 * kB) {
        float v[kB];
#pragma unroll
        for (int t = 0; t < kB; ++t) {
          const int i = i0 + 32 * t;
          v[t] = 0.f;
          if (i < cnt) {
            const int k = i / (nr * ng), rem = i - k * nr * ng, row = rem / ng, c = rem - row * ng;
            v[t] = __ldg(ly.w2_scale + ((size_t)(k ? e1 : e0) * D + r0 + row) * ng + c);
          }
        }
#pragma unroll
        for (int t = 0; t < kB; ++t)
          if (i0 + 32 * t < cnt) dst[i0 + 32 * t] = v[t];
      }
    } else {
      // scales of the gate then up rows: [m][unit j][group c], unit u0 + j of slot (u0 + j) / Hx
      const int ng = D >> g.qgsh, cnt = 2 * nu * ng;
      float* dst = at<float>(g.sm_a + g.q_a_scale);
#pragma unroll 1
      for (int i0 = lane; i0 < cnt; i0 += 32 * kB) {
        float v[kB];
#pragma unroll
        for (int t = 0; t < kB; ++t) {
          const int i = i0 + 32 * t;
          v[t] = 0.f;
          if (i < cnt) {
            const int m = i / (nu * ng), rem = i - m * nu * ng, j = rem / ng, c = rem - j * ng;
            const int u = u0 + j, k = u >= Hx ? 1 : 0;
            v[t] = __ldg((m ? ly.w3_scale : ly.w1_scale) + ((size_t)(k ? e1 : e0) * Hx + u - k * Hx) * ng + c);
          }
        }
#pragma unroll
        for (int t = 0; t < kB; ++t)
          if (i0 + 32 * t < cnt) dst[i0 + 32 * t] = v[t];
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive1(b);
  }
}

// K/V of tokens [ta, ta + n) of head h, layer l -> region K (K rows, then V
// rows at chunk_tok), counted on barrier K (producer warp: lane 0 arms, the
// lanes issue one copy per (block, K or V) segment).
__device__ __noinline__ void tma_kv(int l, int h, int ta, int n) {
  const mie_step_desc& d = ps.d;
  const mie_layer_desc& ly = layer_at(l);
  const int lane = threadIdx.x & 31, bs = d.block_size;
  if (lane == 0) {
    fence_proxy_async_smem();
    bar_arm(kFK, (uint32_t)(2 * n * kHd * 2));
  }
  __syncwarp();
  fence_proxy_async_smem();
  bf16* dst = at<bf16>(ps.g.sm_k);
  const int b0 = ta / bs, b1 = (ta + n - 1) / bs;
#pragma unroll 1
  for (int bi = b0 + lane; bi <= b1; bi += 32) {
    const int tb = max(ta, bi * bs), te = min(ta + n, (bi + 1) * bs);
    int64_t blk = bi;
    if (d.block_table) {
      const int k = bi - cx.blk0;
      const int pb = (k >= 0 && k < kBlkCache) ? blk_s[k] : __ldg(d.block_table + bi);
      if (pb < 0 || pb >= d.num_blocks) set_status(d.status, MIE_ERR_RANGE);
      blk = (pb < 0 || pb >= d.num_blocks) ? 0 : pb;
    }
    const int64_t off = blk * d.kv_stride_block + (int64_t)h * d.kv_stride_head + (int64_t)(tb % bs) * d.kv_stride_tok;
    const uint32_t bytes = (uint32_t)((te - tb) * kHd * 2);
    bulk_copy(dst + (size_t)(tb - ta) * kHd, static_cast<const bf16*>(ly.k_cache) + off, bytes, kFK);
    bulk_copy(dst + (size_t)ps.g.chunk_tok * kHd + (size_t)(tb - ta) * kHd, static_cast<const bf16*>(ly.v_cache) + off,
              bytes, kFK);
  }
}

// LM-head stages [first, first + count) of this CTA's vocab rows into the
// ring over regions A..D (producer lane 0); the rows stay in L2
// preferentially (evict-last), since every step reads them again.
__device__ __noinline__ void tma_head(int first, int count) {
  if ((threadIdx.x & 31) != 0) return;
  const mie_step_desc& d = ps.d;
  const CGeom& g = ps.g;
  int v0, v1;
  split32(d.vocab, blockIdx.x, g.G, &v0, &v1);
  const uint32_t rb = (uint32_t)d.hidden_dim * 2u;
  const int nst = (v1 - v0 + g.head_rows - 1) / g.head_rows;
  fence_proxy_async_smem();
#pragma unroll 1
  for (int i = first; i < first + count && i < nst; ++i) {
    const int slot = i % g.head_stages;
    const int r0 = v0 + i * g.head_rows, n = min(g.head_rows, v1 - r0);
    bar_arm(kFH + slot, (uint32_t)n * rb);
    bulk_copy(at<uint8_t>(g.sm_k) + (size_t)slot * g.head_rows * rb,
              static_cast<const uint8_t*>(d.embedding) + (size_t)r0 * rb, (uint32_t)n * rb, kFH + slot, true);
  }
}

// ---------------------------------------------------------------------------
// Compute routines
// ---------------------------------------------------------------------------
// out[r] = rows[r] . x for r < n: bf16 rows of nvec 16-byte vectors (<= 96)
// staged in shared memory, x fp32 in shared memory (rows [split, n) dot x1
// when x1 is set).  Consumer warp w forms rows w, w + kCW, ...: R rows per iteration,
// one partial sum per 16-byte vector and row.  No barrier.
template <int R>
__device__ __forceinline__ void gemv_rows(const uint4* rows, int n, int nvec, const float* xr, const float* xr1,
                                          int split, float* out) {
  constexpr int NV = Seg<bf16>::kNV;
  const int lane = threadIdx.x & 31;
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll 1
  for (int r = threadIdx.x >> 5; r < n; r += R * kCW) {
    uint4 w[R][NV];
#pragma unroll
    for (int k = 0; k < R; ++k) {
      const int rk = r + k * kCW < n ? r + k * kCW : r;
      const uint4* rp = rows + (size_t)rk * nvec;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int v = lane + kWarp * j;
        w[k][j] = v < nvec ? rp[v] : z;
      }
    }
    float sum[R];
#pragma unroll
    for (int k = 0; k < R; ++k) {
      const float* x = (xr1 && r + k * kCW >= split) ? xr1 : xr;
      sum[k] = 0.f;
#pragma unroll
      for (int j = 0; j < NV; ++j) sum[k] += dot_vec(w[k][j], x + j * kPV, 0.f, (const bf16*)nullptr);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
      for (int k = 0; k < R; ++k) sum[k] += __shfl_xor_sync(0xffffffffu, sum[k], o);
    }
    if (lane == 0) {
#pragma unroll
      for (int k = 0; k < R; ++k)
        if (r + k * kCW < n) out[r + k * kCW] = sum[k];
    }
  }
}
// int8 rows staged in shared memory (nw 32-bit words of four values each,
// the values' fp32 group scales [row][ngr] at sc, group = 1 << gsh): out[r] =
// sum over the row's words of scale x (q . x), x fp32 in registers (lane l
// holds x of its words l, l + 32, ... : xr[4k + j] = x[4 (l + 32 k) + j]).
// Consumer warp w forms rows w, w + kCW, ...: R rows per iteration.  Rows
// [split, n) use xr1.  The values are two's complement; flipping the sign
// bits offsets them to unsigned for byte_to_f.
constexpr int kQ8Words = 6;  // words per lane of a row of <= 768 int8 values
template <int R>
__device__ __forceinline__ void gemv_q8_rows(const uint32_t* rows, const float* sc, int n, int nw, int ngr, int gsh,
                                             const float* xr, const float* xr1, int split, float* out) {
  const int lane = threadIdx.x & 31;
#pragma unroll 1
  for (int r = threadIdx.x >> 5; r < n; r += R * kCW) {
    uint32_t w[R][kQ8Words];
    float s[R][kQ8Words];
#pragma unroll
    for (int k = 0; k < R; ++k) {
      const int rk = r + k * kCW < n ? r + k * kCW : r;
#pragma unroll
      for (int j = 0; j < kQ8Words; ++j) {
        const int wi = lane + 32 * j;
        w[k][j] = wi < nw ? rows[(size_t)rk * nw + wi] ^ 0x80808080u : 0x80808080u;  // 0x80808080: four zeros
        s[k][j] = wi < nw ? sc[(size_t)rk * ngr + ((4 * wi) >> gsh)] : 0.f;
      }
    }
    float sum[R];
#pragma unroll
    for (int k = 0; k < R; ++k) {
      const float* x = (xr1 && r + k * kCW >= split) ? xr1 : xr;
      sum[k] = 0.f;
#pragma unroll
      for (int j = 0; j < kQ8Words; ++j) {
        float part = byte_to_f(w[k][j], 0x7440u) * x[4 * j];
        part = fmaf(byte_to_f(w[k][j], 0x7441u), x[4 * j + 1], part);
        part = fmaf(byte_to_f(w[k][j], 0x7442u), x[4 * j + 2], part);
        part = fmaf(byte_to_f(w[k][j], 0x7443u), x[4 * j + 3], part);
        sum[k] = fmaf(part, s[k][j], sum[k]);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
      for (int k = 0; k < R; ++k) sum[k] += __shfl_xor_sync(0xffffffffu, sum[k], o);
    }
    if (lane == 0) {
#pragma unroll
      for (int k = 0; k < R; ++k)
        if (r + k * kCW < n) out[r + k * kCW] = sum[k];
    }
  }
}
__device__ __forceinline__ void load_xq_regs(float* xr, const float* x, int nw) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < kQ8Words; ++j) {
    const int wi = lane + 32 * j;
    const float4 v = wi < nw ? *reinterpret_cast<const float4*>(x + 4 * wi) : make_float4(0.f, 0.f, 0.f, 0.f);
    xr[4 * j] = v.x;
    xr[4 * j + 1] = v.y;
    xr[4 * j + 2] = v.z;
    xr[4 * j + 3] = v.w;
  }
}
// GEMV of n staged int8 rows (rows [split, n) dot x1 when x1 is set).
__device__ __noinline__ void gemv_q8(const uint32_t* rows, const float* sc, int n, int nw, int ngr, int gsh,
                                     const float* x, float* out, const float* x1 = nullptr, int split = 0) {
  if ((int)(threadIdx.x >> 5) >= n) return;
  float xr[4 * kQ8Words];
  if (x1) {
    // rows [split, n) dot x1 (n <= kCW: one row per warp)
    load_xq_regs(xr, (int)(threadIdx.x >> 5) >= split ? x1 : x, nw);
    gemv_q8_rows<1>(rows, sc, n, nw, ngr, gsh, xr, nullptr, 0, out);
    return;
  }
  load_xq_regs(xr, x, nw);
  if (n > 2 * kCW) {
    gemv_q8_rows<3>(rows, sc, n, nw, ngr, gsh, xr, nullptr, 0, out);
  } else {
    gemv_q8_rows<2>(rows, sc, n, nw, ngr, gsh, xr, nullptr, 0, out);
  }
}

// GEMV of n staged rows (rows [split, n) dot x1 when x1 is set).
__device__ __noinline__ void gemv(const uint4* rows, int n, int nvec, const float* x, float* out,
                                  const float* x1 = nullptr, int split = 0) {
  constexpr int NV = Seg<bf16>::kNV;
  if ((int)(threadIdx.x >> 5) >= n) return;
  float xr[NV * kPV];
  if (x1) {
    // rows [split, n) dot x1 (n <= kCW: one row per warp, so each warp loads
    // the one vector its row needs)
    load_x_regs<bf16>(xr, (int)(threadIdx.x >> 5) >= split ? x1 : x, nvec);
    gemv_rows<1>(rows, n, nvec, xr, nullptr, 0, out);
    return;
  }
  load_x_regs<bf16>(xr, x, nvec);
  if (n > 3 * kCW) {
    gemv_rows<4>(rows, n, nvec, xr, nullptr, 0, out);  // LM-head stages: up to 60 rows in one pass
  } else if (n > 2 * kCW) {
    gemv_rows<3>(rows, n, nvec, xr, nullptr, 0, out);  // up to 45 rows in one pass
  } else {
    gemv_rows<2>(rows, n, nvec, xr, nullptr, 0, out);
  }
}

// Online softmax of q over this split's old tokens [t0, t1) in chunks of
// chunk_tok (the first chunk was staged ahead).  Leaves (acc [hd], m, l) at
// `res` (acc, then m, l).  q fp32 in shared memory.
__device__ __noinline__ bool att_core(bool ok, int l, int h, int t0, int t1, const float* q, float* res) {
  const mie_step_desc& d = ps.d;
  const CGeom& g = ps.g;
  const int tid = threadIdx.x, chunk = g.chunk_tok;
  constexpr int VPH = kHd / kPV;           // 16-byte pieces per K row
  constexpr int Gp = kCT / kHd;            // PV groups (threads past Gp * hd idle)
  const int gi = tid / kHd, dc = tid % kHd;
  const bf16* ks = at<const bf16>(g.sm_k);
  const bf16* vs = ks + (size_t)chunk * kHd;
  float* sc = at<float>(g.sm_sc);
  float* pv = at<float>(g.sm_ab);  // [Gp][hd]
  const float scale = d.attn_scale;
  float m_run = -INFINITY, l_run = 0.f, acc = 0.f;
  const int nch = (t1 - t0 + chunk - 1) / chunk;
#pragma unroll 1
  for (int ci = 0; ci < nch; ++ci) {
    const int ta = t0 + ci * chunk, n = min(chunk, t1 - ta);
    if (ci > 0) {
      csync();  // the previous chunk is no longer read
      if (ok) issue_kv(cons_side(), kFK2, l, h, ta, n);
    }
    ok = bwait(ok, ci == 0 ? kFK : kFK2);
    CSTAMP(l, 16);
    float mloc = -INFINITY;
    if (ok) {
#pragma unroll 1
      for (int t = tid; t < n; t += kCT) {
        const uint4* kr = reinterpret_cast<const uint4*>(ks + (size_t)t * kHd);
        // the start piece rotates with t: the threads of a warp read distinct banks
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
        for (int jj = 0; jj < VPH; jj += 4) {
          const int j0 = (jj + t) & (VPH - 1), j1 = (jj + 1 + t) & (VPH - 1);
          const int j2 = (jj + 2 + t) & (VPH - 1), j3 = (jj + 3 + t) & (VPH - 1);
          a0 = dot_vec(kr[j0], q + j0 * kPV, a0, (const bf16*)nullptr);
          a1 = dot_vec(kr[j1], q + j1 * kPV, a1, (const bf16*)nullptr);
          a2 = dot_vec(kr[j2], q + j2 * kPV, a2, (const bf16*)nullptr);
          a3 = dot_vec(kr[j3], q + j3 * kPV, a3, (const bf16*)nullptr);
        }
        const float v = ((a0 + a1) + (a2 + a3)) * scale;
        sc[t] = v;
        mloc = fmaxf(mloc, v);
      }
    }
    mloc = warp_max(mloc);
    if ((tid & 31) == 0) red_s[tid >> 5] = mloc;
    ok = !csync_or(!ok);  // CTA-uniform: the next chunk's copies need every consumer thread
    float bmax = -INFINITY;
#pragma unroll
    for (int i = 0; i < kCW; ++i) bmax = fmaxf(bmax, red_s[i]);
    const float mn = fmaxf(m_run, bmax);
    CSTAMP(l, 17);
    const float alpha = m_run == -INFINITY ? 0.f : expf(m_run - mn);
    float ls = 0.f;
    if (ok) {
#pragma unroll 1
      for (int t = tid; t < n; t += kCT) {
        const float p = expf(sc[t] - mn);
        sc[t] = p;
        ls += p;
      }
    }
    ls = warp_sum(ls);
    if ((tid & 31) == 0) red2_s[tid >> 5] = ls;
    csync();  // also orders the probabilities before the PV reads
    float bsum = 0.f;
#pragma unroll
    for (int i = 0; i < kCW; ++i) bsum += red2_s[i];
    l_run = l_run * alpha + bsum;
    m_run = mn;
    CSTAMP(l, 18);
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    if (ci == 0 && gi == Gp) {
      // the warp past the PV groups: scale * q . k_new (q, k_new gathered before
      // the core), for the merge
      const int lane = tid & 31;
      float p = q[lane] * q[kHd + lane] + q[lane + 32] * q[kHd + lane + 32];
      p = warp_sum(p);
      if (lane == 0) cx.snew = p * scale;
    }
    if (ok && gi < Gp) {
      int t = gi;
#pragma unroll 1
      for (; t + 3 * Gp < n; t += 4 * Gp) {
        a0 = fmaf(sc[t], __bfloat162float(vs[(size_t)t * kHd + dc]), a0);
        a1 = fmaf(sc[t + Gp], __bfloat162float(vs[(size_t)(t + Gp) * kHd + dc]), a1);
        a2 = fmaf(sc[t + 2 * Gp], __bfloat162float(vs[(size_t)(t + 2 * Gp) * kHd + dc]), a2);
        a3 = fmaf(sc[t + 3 * Gp], __bfloat162float(vs[(size_t)(t + 3 * Gp) * kHd + dc]), a3);
      }
#pragma unroll 1
      for (; t < n; t += Gp) a0 = fmaf(sc[t], __bfloat162float(vs[(size_t)t * kHd + dc]), a0);
    }
    acc = fmaf(acc, alpha, (a0 + a1) + (a2 + a3));
    CSTAMP(l, 19);
  }
  if (nch == 0 && gi == Gp) {
    const int lane = tid & 31;
    float p = q[lane] * q[kHd + lane] + q[lane + 32] * q[kHd + lane + 32];
    p = warp_sum(p);
    if (lane == 0) cx.snew = p * scale;
  }
  csync();  // every chunk read (the K/V region may be restaged), scores scratch free
  if (gi < Gp) pv[gi * kHd + dc] = acc;
  csync();
  if (tid < kHd) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < Gp; ++k) s += pv[k * kHd + tid];
    res[tid] = s;
  } else if (tid == kHd) {
    res[kHd] = m_run;
    res[kHd + 1] = l_run;
  }
  csync();
  return ok;
}

// ---------------------------------------------------------------------------
// ATT: attention of layer l for the attention clusters (see the file comment)
// ---------------------------------------------------------------------------
template <bool EP>
__device__ __noinline__ bool att_phase(const CStepParams& P, int l, bool ok) {
  const mie_step_desc& d = ps.d;
  const CGeom& g = ps.g;
  const mie_layer_desc& ly = layer_at(l);
  const int tid = threadIdx.x, D = d.hidden_dim, nvD = D / kPV, par = l & 1;
  const uint32_t tag = tag_of(l);
  const int pos = cx.pos;
  const Split a = split_of(pos);
  float* xs = at<float>(g.sm_x);
  float* xn = at<float>(g.sm_xn);
  CSTAMP(l, 0);
  ok = bwait(ok, kFR);  // the layer's norm weights (and router)
  CSTAMP(l, 12);
  // ---- x: the token embedding (layer 0) or exchange X ----
  // RMSNorm folded in: the thread that received element i forms x_i * nw_i
  // and its share of the square sum (the poll gives thread t the elements
  // t, t + kCT, ...), so the block sum needs no barrier of its own; the
  // q/k/v GEMV runs on x * nw and its results are scaled by rs.
  int bad = 0;
  if (l == 0) {
    const bf16* e = static_cast<const bf16*>(d.embedding) + cx.tok * D;
#pragma unroll 1
    for (int i = tid; i < D; i += kCT) xs[i] = __bfloat162float(e[i]);
  } else if (ok) {
    bad = EP ? poll_ranks(l, D, at<const float>(g.sm_xm) + (size_t)((l - 1) & 1) * D, xs, 0)
             : poll(g.ll + g.off_x[par], D, tag, xs, Ident{});
  }
  {
    const bf16* nw = at<const bf16>(g.sm_r) + (size_t)d.num_experts * D;
    float s2 = 0.f;
#pragma unroll 1
    for (int i = tid; i < D; i += kCT) {
      const float x = xs[i];
      s2 = fmaf(x, x, s2);
      xn[i] = x * __bfloat162float(nw[i]);
    }
    s2 = warp_sum(s2);
    if ((tid & 31) == 0) red_s[tid >> 5] = s2;
  }
  ok = !csync_or(bad || !ok);
  float rs;
  {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < kCW; ++i) t += red_s[i];
    rs = rsqrtf(t / (float)D + d.eps);
  }
  CSTAMP(l, 1);
  // ---- this split's q, k, v rows ----
  ok = bwait(ok, kFQ);
  CSTAMP(l, 14);
  float* qo = at<float>(g.sm_qkv);
  const int nrows = 4 * a.np + a.nv;
  if (ok) gemv(at<const uint4>(g.sm_a), nrows, nvD, xn, qo);
  csync();
  CSTAMP(l, 2);
  // ---- RoPE, cache store, send q / k_new / v_new to every CTA of the cluster ----
  float* gq = at<float>(g.sm_g) + (size_t)par * 3 * kHd;  // [q | k | v] of this layer parity
  const float* cs = d.rope_cos + (int64_t)pos * (kHd / 2);
  const float* sn = d.rope_sin + (int64_t)pos * (kHd / 2);
  const int64_t slot = cx.slot + (int64_t)a.h * d.kv_stride_head;
  if (ok) {
    int dim = -1, dim2 = -1;
    float v1 = 0.f, v2 = 0.f;
    if (tid < a.np) {  // q pair
      const int i = a.p0 + tid;
      const float x1 = qo[tid] * rs, x2 = qo[a.np + tid] * rs;
      v1 = x1 * cs[i] - x2 * sn[i];
      v2 = x2 * cs[i] + x1 * sn[i];
      dim = i;
      dim2 = i + kHd / 2;
    } else if (tid >= 64 && tid < 64 + a.np) {  // k pair: rounded to the cache type, stored
      const int k = tid - 64, i = a.p0 + k;
      const float x1 = qo[2 * a.np + k] * rs, x2 = qo[3 * a.np + k] * rs;
      const bf16 k1 = __float2bfloat16_rn(x1 * cs[i] - x2 * sn[i]);
      const bf16 k2 = __float2bfloat16_rn(x2 * cs[i] + x1 * sn[i]);
      bf16* kc = static_cast<bf16*>(ly.k_cache);
      kc[slot + i] = k1;
      kc[slot + i + kHd / 2] = k2;
      v1 = __bfloat162float(k1);
      v2 = __bfloat162float(k2);
      dim = kHd + i;
      dim2 = kHd + i + kHd / 2;
    } else if (tid >= 128 && tid < 128 + a.nv) {  // v row
      const int k = tid - 128, i = a.v0 + k;
      const bf16 vv = __float2bfloat16_rn(qo[4 * a.np + k] * rs);
      static_cast<bf16*>(ly.v_cache)[slot + i] = vv;
      v1 = __bfloat162float(vv);
      dim = 2 * kHd + i;
    }
    if (dim >= 0) {
#pragma unroll 1
      for (int r = 0; r < kCS; ++r) {
        dsmem_st(dsmem_addr(gq + dim, (uint32_t)r), v1);
        if (dim2 >= 0) dsmem_st(dsmem_addr(gq + dim2, (uint32_t)r), v2);
      }
    }
  }
  CSTAMP(l, 15);
  cluster_sync_all();  // cluster barrier 1: q, k_new, v_new of the head complete in every CTA

  CSTAMP(l, 3);
  // ---- attention over the old tokens ----
  float* mg = at<float>(g.sm_mg) + (size_t)par * kCS * kMg;  // [CS][acc, m, l]
  float* mine = at<float>(g.sm_ov);                          // this split's result, then o
  ok = att_core(ok, l, a.h, a.t0, a.t1, gq, mine);
  CSTAMP(l, 4);
  // region K is free: the producer stages the next layer's first K/V chunk
  if (l + 1 < d.num_layers) region_free(kEK);
  CSTAMP(l, 21);
  if (ok && tid < kHd + 2) {
    const float v = mine[tid];
    float* dst = mg + (size_t)a.s * kMg + tid;
#pragma unroll 1
    for (int r = 0; r < kCS; ++r) dsmem_st(dsmem_addr(dst, (uint32_t)r), v);
  }
  CSTAMP(l, 22);
  cluster_sync_all();  // cluster barrier 2: every split's (acc, m, l)
  CSTAMP(l, 5);
  // ---- merge: o_h = (sum_s e^(m_s - M) acc_s + e^(s_new - M) v_new) / (sum_s e^(m_s - M) l_s + e^(s_new - M)) ----
  float* ov = mine;  // [hd]: the split result is no longer needed
  if (tid < kHd) {
    const float snew = cx.snew;
    float M = snew;
#pragma unroll
    for (int s = 0; s < kCS; ++s) M = fmaxf(M, mg[s * kMg + kHd]);
    const float wn = expf(snew - M);
    float num = wn * gq[2 * kHd + tid], den = wn;
#pragma unroll
    for (int s = 0; s < kCS; ++s) {
      const float ms = mg[s * kMg + kHd];
      const float w = ms == -INFINITY ? 0.f : expf(ms - M);
      num = fmaf(w, mg[s * kMg + tid], num);
      den = fmaf(w, mg[s * kMg + kHd + 1], den);
    }
    ov[tid] = num / den;
  }
  csync();
  CSTAMP(l, 23);
  // ---- out_proj partial of head h: rows [r0, r0 + nr) . o_h -> exchange P[h] ----
  ok = bwait(ok, kFO);
  CSTAMP(l, 24);
  if (ok) {
    // 8 lanes per row (8 bf16 each), 4 rows per warp per pass
    const int lane = tid & 31, sub = lane >> 3, e = lane & 7;
    const uint4* tile = at<const uint4>(g.sm_o);
    float o8[kPV];
#pragma unroll
    for (int j = 0; j < kPV; ++j) o8[j] = ov[e * kPV + j];
    uint64_t* pw = g.ll + g.off_p[par] + (int64_t)a.h * D + a.r0;
    // every lane of a warp takes the same number of passes (the shuffles)
#pragma unroll 1
    for (int rw = (tid >> 5) * 4; rw < a.nr; rw += kCW * 4) {
      const int r = rw + sub;
      float s = r < a.nr ? dot_vec(tile[r * (kHd / kPV) + e], o8, 0.f, (const bf16*)nullptr) : 0.f;
      s += __shfl_xor_sync(0xffffffffu, s, 4);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      if (e == 0 && r < a.nr) ll_put(pw + r, s, tag);
    }
  }
  csync();  // the tile is no longer read
  CSTAMP(l, 25);
  if (l + 1 < d.num_layers) region_free(kEO);
  CSTAMP(l, 6);
  return ok;
}

// Routing of layer l after cluster barrier 3, by one full warp (every
// consumer warp and the producer warp compute the same bits): the RMSNorm
// scale rs of x_mid from the cluster's square sums and the top-2 experts from
// the cluster's router partials, both summed in rank order.  One expert per
// lane (E <= 32): lane e holds expert e's logit (its partials' sum times rs;
// NaN ranks as -inf).  (value, lower id) is a total order, so the butterfly
// gives every lane the same answer: the maximum with ties to the lower id,
// then the maximum of the others with ties to the lower id -- the repeated
// argmax of the reference's router (src/moe_engine/fused_moe.py:143-150).
struct Route {
  float rs;        // RMSNorm scale of x_mid
  int sel0, sel1;  // the experts
  float bv, cv;    // and their logits
};
// RMSNorm scale of layer l's x_mid from the cluster's square sums.
__device__ __forceinline__ float xmid_scale(int l) {
  const float* ssb = at<const float>(ps.g.sm_ss) + (size_t)(l & 1) * kCS;
  float t = 0.f;
#pragma unroll
  for (int s = 0; s < kCS; ++s) t += ssb[s];
  return rsqrtf(t / (float)ps.d.hidden_dim + ps.d.eps);
}
__device__ __forceinline__ Route route_top2(int l) {
  const mie_step_desc& d = ps.d;
  const int E = d.num_experts, par = l & 1, lane = threadIdx.x & 31;
  const float* rps = at<const float>(ps.g.sm_rp) + (size_t)par * kCS * E;
  Route r;
  r.rs = xmid_scale(l);
  float lv = -INFINITY;
  if (lane < E) {
    float q = 0.f;
#pragma unroll
    for (int s = 0; s < kCS; ++s) q += rps[s * E + lane];
    lv = r.rs * q;
    if (lv != lv) lv = -INFINITY;
  }
  r.bv = lv;
  r.sel0 = lane;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, r.bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, r.sel0, o);
    if (better(ov, oi, r.bv, r.sel0)) {
      r.bv = ov;
      r.sel0 = oi;
    }
  }
  r.cv = lane == r.sel0 ? -INFINITY : lv;
  r.sel1 = lane == r.sel0 ? 64 : lane;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, r.cv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, r.sel1, o);
    if (better(ov, oi, r.cv, r.sel1)) {
      r.cv = ov;
      r.sel1 = oi;
    }
  }
  return r;
}
// The slots' experts in this rank's weight stack (expert parallel: -1 for a
// slot held by another rank).
template <bool EP>
__device__ __forceinline__ void local_experts(int sel0, int sel1, int* le0, int* le1) {
  *le0 = sel0;
  *le1 = sel1;
  if (EP) {
    const mie_step_desc& d = ps.d;
    *le0 = (unsigned)(sel0 - d.expert_base) < (unsigned)d.expert_count ? sel0 - d.expert_base : -1;
    *le1 = (unsigned)(sel1 - d.expert_base) < (unsigned)d.expert_count ? sel1 - d.expert_base : -1;
  }
}

// ---------------------------------------------------------------------------
// MOE: x_mid, routing, the two selected experts, x of layer l + 1
// ---------------------------------------------------------------------------
template <bool EP, bool Q8>
__device__ __noinline__ bool moe_phase(const CStepParams& P, int l, bool ok, bool att) {
  const mie_step_desc& d = ps.d;
  const CGeom& g = ps.g;
  const int tid = threadIdx.x, D = d.hidden_dim, Hx = d.expert_hidden_dim, E = d.num_experts, H = d.num_heads;
  const int nvD = D / kPV, nvH = Hx / kPV, par = l & 1;
  const uint32_t tag = tag_of(l);
  const Split a = split_of(cx.pos);
  float* xs = at<float>(g.sm_x);
  float* xn = at<float>(g.sm_xn);
  float* xm = at<float>(g.sm_xm) + (size_t)par * D;
  float* ssb = at<float>(g.sm_ss) + (size_t)par * kCS;
  float* rps = at<float>(g.sm_rp) + (size_t)par * kCS * E;  // [CS][E] router partials
  float* pr = at<float>(g.sm_pr);  // [H][nr] partials, then [nr] x rows (non-attention CTAs)
  float* ab = at<float>(g.sm_ab);
  float* hb = at<float>(g.sm_h);
  // ---- receive rows [r0, r0 + nr) of every head's partial (and of x) ----
  const int nr = a.nr, r0 = a.r0;
  const bool need_x = !att && l > 0;
  constexpr bool ep = EP;
  {
    // expert parallel: x's rows come from the cross-GPU exchange below
    const int n = H * nr + (need_x && !ep ? nr : 0);
    const uint64_t* pb = g.ll + g.off_p[par];
    const int64_t xoff = g.off_x[par] - g.off_p[par];
    int bad = 0;
    if (ok)
      bad = poll(pb, n, tag, pr, [=](int i) -> int {
        if (i < H * nr) {
          const int h = i / nr;
          return h * D + r0 + (i - h * nr);
        }
        return (int)xoff + r0 + (i - H * nr);
      });
    if (ok && need_x && ep && !bad)
      bad = poll_ranks(l, nr, at<const float>(g.sm_xm) + (size_t)((l - 1) & 1) * D, pr + (size_t)H * nr, r0);
    if (!att && l == 0) {
      const bf16* e = static_cast<const bf16*>(d.embedding) + cx.tok * D;
      for (int i = tid; i < nr; i += kCT) pr[H * nr + i] = __bfloat162float(e[r0 + i]);
    }
    ok = !csync_or(bad || !ok);
  }
  CSTAMP(l, 26);
  // ---- x_mid rows, their square sum and their router partials -> every CTA of the cluster ----
  // The router logit of expert e is rs * sum_i (x_mid_i * nw_i) * w_e,i with
  // rs the RMSNorm scale: each CTA sends the partial dots of its rows, and
  // routing right after the cluster barrier needs no pass over D.
  if (!att) ok = bwait(ok, kFR);  // router rows + norm weights (the attention CTAs waited already)
  const bf16* rw = at<const bf16>(g.sm_r);
  const bf16* nw = rw + (size_t)(E + 1) * D;
  float v = 0.f;
  if (tid < nr) {
    v = att ? xs[r0 + tid] : pr[H * nr + tid];
#pragma unroll 1
    for (int h = 0; h < H; ++h) v += pr[h * nr + tid];
    ab[tid] = v * __bfloat162float(nw[r0 + tid]);
  }
  float s2 = warp_sum(v * v);  // rows beyond nr contribute 0
  if ((tid & 31) == 0) red_s[tid >> 5] = s2;
  csync();
  if (ok) {
    const int warp = tid >> 5, lane = tid & 31;
    if (tid < nr) {
#pragma unroll 1
      for (int r = 0; r < kCS; ++r) dsmem_st(dsmem_addr(xm + r0 + tid, (uint32_t)r), v);
    } else if (tid >= kCT - 32 && tid - (kCT - 32) < kCS) {
      float t = 0.f;
#pragma unroll
      for (int i = 0; i < kCW; ++i) t += red_s[i];
      dsmem_st(dsmem_addr(ssb + a.s, (uint32_t)(tid - (kCT - 32))), t);
    }
    // router partials of this CTA's rows: expert e on warp kCW - 1 - e (mod
    // kCW), away from the row senders of the low warps
#pragma unroll 1
    for (int e = kCW - 1 - warp; e < E; e += kCW) {
      const bf16* we = rw + (size_t)e * D + r0;
      float p = 0.f;
#pragma unroll 1
      for (int i = lane; i < nr; i += 32) p = fmaf(ab[i], __bfloat162float(we[i]), p);
      p = warp_sum(p);
      if (lane < kCS) dsmem_st(dsmem_addr(rps + a.s * E + e, (uint32_t)lane), p);
    }
  }
  CSTAMP(l, 27);
  cluster_sync_all();  // cluster barrier 3: x_mid and the router partials complete in every CTA
  CSTAMP(l, 7);
  // ---- routing: the producer warp computes it at once and stages the
  // selected experts' rows.  The consumers need the RMSNorm scale now and the
  // routing weights only for the combine, so they route while the expert
  // hidden units are exchanged -- except with expert parallelism, where the
  // up units need to know which slots this rank holds. ----
  Route rt;
  unsigned held = 3u;  // the slots this rank computes
  if constexpr (EP) {
    rt = route_top2(l);
    int le0, le1;
    local_experts<EP>(rt.sel0, rt.sel1, &le0, &le1);
    held = (le0 >= 0 ? 1u : 0u) | (le1 >= 0 ? 2u : 0u);
  }
  float rs;
  if constexpr (EP)
    rs = rt.rs;
  else
    rs = xmid_scale(l);
  CSTAMP(l, 28);
  CSTAMP(l, 30);
  // the normalised x_mid for the up GEMV, while the expert rows are in flight
#pragma unroll 1
  for (int i = tid; i < D; i += kCT) xn[i] = (xm[i] * rs) * __bfloat162float(nw[i]);
  csync();  // router rows and norm weights read: region R may be restaged; xn complete
  region_free(kER);  // the producer stages the next layer's router + norms, or the final norm
  CSTAMP(l, 8);
  // ---- up units: silu(gate) * up -> exchange H ----
  int u0, u1, q0, q1;
  split32(2 * Hx, blockIdx.x, g.G, &u0, &u1);
  split32(D, blockIdx.x, g.G, &q0, &q1);
  const int nu = u1 - u0, nq = q1 - q0;
  ok = bwait(ok, kFE);
  CSTAMP(l, 31);
  if (ok) {
    if constexpr (Q8)
      gemv_q8(at<const uint32_t>(g.sm_a), at<const float>(g.sm_a + g.q_a_scale), 2 * nu, D / 4, D >> g.qgsh,
              g.qgsh, xn, ab);
    else
      gemv(at<const uint4>(g.sm_a), 2 * nu, nvD, xn, ab);
  }
  csync();  // region A no longer read
  if (ok && tid < nu) {
    float h = silu(ab[tid]) * ab[nu + tid];
    // a slot held by another rank: its rows were not staged, its units are 0
    if (EP && !(held >> (u0 + tid < Hx ? 0 : 1) & 1u)) h = 0.f;
    ll_put(g.ll + g.off_h[par] + u0 + tid, h, tag);
  }
  if (att && l + 1 < d.num_layers) region_free(kEA);  // the producer stages the next layer's q/k/v rows
  if constexpr (!EP) rt = route_top2(l);
  const float e1 = expf(rt.cv - rt.bv);
  const float wt0 = 1.0f / (1.0f + e1), wt1 = e1 / (1.0f + e1);
  CSTAMP(l, 9);
  // ---- down rows of both slots . h + residual -> exchange X of layer l + 1 ----
  {
    int bad = 0;
    if (ok) bad = poll(g.ll + g.off_h[par], 2 * Hx, tag, hb, Ident{});
    ok = !csync_or(bad || !ok);
  }
  CSTAMP(l, 10);
  ok = bwait(ok, kFD);
  CSTAMP(l, 13);
  if (ok) {
    if constexpr (Q8)
      gemv_q8(at<const uint32_t>(g.sm_d), at<const float>(g.sm_d + g.q_d_scale), 2 * nq, Hx / 4, Hx >> g.qgsh,
              g.qgsh, hb, ab, hb + Hx, nq);
    else
      gemv(at<const uint4>(g.sm_d), 2 * nq, nvH, hb, ab, hb + Hx, nq);
  }
  csync();  // region D no longer read
  CSTAMP(l, 20);
  if (ok && tid < nq) {
    const int r = q0 + tid;
    if constexpr (EP) {
      // this rank's partial: its slots in slot order (the per-layer kernels'
      // combine); the readers add x_mid
      float y = 0.f;
      if (held & 1u) y = fmaf(wt0, ab[tid], y);
      if (held & 2u) y = fmaf(wt1, ab[nq + tid], y);
      peer_put(l + 1, r, y);
    } else {
      const float y = fmaf(wt1, ab[nq + tid], fmaf(wt0, ab[tid], xm[r]));
      ll_put(g.ll + g.off_x[(l + 1) & 1] + r, y, tag_of(l + 1));
      if (l == d.num_layers - 1) d.x[r] = y;
    }
  }
  // after the last layer the ring area is free (x_mid, read just above, lies
  // in it too): the producer starts the LM-head ring
  if (l == d.num_layers - 1) {
    if (EP) {  // the head adds the ranks' partials to x_mid: keep it outside the ring
      float* xs = at<float>(g.sm_x);
#pragma unroll 1
      for (int i = tid; i < D; i += kCT) xs[i] = xm[i];
    }
    csync();
    region_free(kED);
  }
  if (tid == 0) {
    cx.sel0 = rt.sel0;
    cx.sel1 = rt.sel1;
  }
  CSTAMP(l, 11);
  return ok;
}

// ---------------------------------------------------------------------------
// HEAD: final norm -> tied LM head -> argmax + device bookkeeping
// ---------------------------------------------------------------------------
__device__ __noinline__ void head_finish(int bi) {
  const mie_step_desc& d = ps.d;
  if (bi < 0 || bi >= d.vocab) {  // every logit NaN
    set_status(d.status, MIE_ERR_RANGE);
    bi = 0;
  }
  *d.token = bi;
  *d.pos = cx.pos + 1;
  if (d.tokens_log && d.log_count) {
    const int k = cx.log_k;
    if (k < d.log_capacity) d.tokens_log[k] = bi;
    *d.log_count = k + 1;
  }
  if (d.done && bi == d.eos_id) *d.done = 1;
  *d.lm_counter = 0u;
  if (ps.g.peer_world > 1) *reinterpret_cast<volatile uint32_t*>(ps.g.peer_seq) = cx.pstep;
  __threadfence();
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(ps.g.ll + kHdrStep), "l"((uint64_t)cx.step) : "memory");
}

template <bool EP>
__device__ __noinline__ bool head_phase(bool ok) {
  const mie_step_desc& d = ps.d;
  const CGeom& g = ps.g;
  const int G = g.G, c = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int D = d.hidden_dim, nvD = D / kPV, L = d.num_layers;
  float* xs = at<float>(g.sm_x);
  float* xn = at<float>(g.sm_xn);
  float* ab = at<float>(g.sm_ab);
  CSTAMP(L, 0);
  ok = bwait(ok, kFR);  // the final norm weights
  // the final RMSNorm folded into the receive as in the attention phase: the
  // LM-head GEMV runs on x * w, its logits are scaled by rs
  float rs;
  {
    int bad = 0;
    if (ok) bad = EP ? poll_ranks(L, D, xs, xs, 0) : poll(g.ll + g.off_x[L & 1], D, tag_of(L), xs, Ident{});
    const bf16* fw = at<const bf16>(g.sm_fn);
    float s2 = 0.f;
#pragma unroll 1
    for (int i = tid; i < D; i += kCT) {
      const float x = xs[i];
      s2 = fmaf(x, x, s2);
      xn[i] = x * __bfloat162float(fw[i]);
    }
    s2 = warp_sum(s2);
    if ((tid & 31) == 0) red_s[tid >> 5] = s2;
    ok = !csync_or(bad || !ok);
    if (EP && ok && c == 0) {  // x after the last layer (the row owners hold only their partials)
#pragma unroll 1
      for (int i = tid; i < D; i += kCT) d.x[i] = xs[i];
    }
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < kCW; ++i) t += red_s[i];
    rs = rsqrtf(t / (float)D + d.eps);
  }
  CSTAMP(L, 1);
  int v0, v1;
  split32(d.vocab, c, G, &v0, &v1);
  const int nst = (v1 - v0 + g.head_rows - 1) / g.head_rows;
  float best_v = -INFINITY;
  int best_i = 0x7fffffff;
#pragma unroll 1
  for (int i = 0; i < nst; ++i) {
    const int slot = i % g.head_stages;
    ok = bwait(ok, kFH + slot);
    const int r0 = v0 + i * g.head_rows, n = min(g.head_rows, v1 - r0);
    if (ok) gemv(at<const uint4>(g.sm_k) + (size_t)slot * g.head_rows * nvD, n, nvD, xn, ab);
    csync();  // stage no longer read, ab complete
    if (i + g.head_stages < nst) region_free(kEH + slot);  // the producer refills the slot
    if (tid < n) {
      const float v = ab[tid] * rs;
      const int row = r0 + tid;
      if (d.logits) d.logits[row] = v;
      if (better(v, row, best_v, best_i)) {
        best_v = v;
        best_i = row;
      }
    }
  }
  CSTAMP(L, 2);
  ok = !csync_or(!ok);  // CTA-uniform before the CTA argmax and its barriers
  if (!ok) return false;
  // CTA argmax: (value, lower index) is a total order
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
    if (better(ov, oi, best_v, best_i)) {
      best_v = ov;
      best_i = oi;
    }
  }
  if (lane == 0) {
    bestv_s[warp] = best_v;
    besti_s[warp] = best_i;
  }
  csync();
  if (tid == 0) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll 1
    for (int w = 0; w < kCW; ++w)
      if (better(bestv_s[w], besti_s[w], bv, bi)) {
        bv = bestv_s[w];
        bi = besti_s[w];
      }
    d.lm_partial_val[c] = bv;
    d.lm_partial_idx[c] = bi;
    cx.last = atom_add_acq_rel_gpu(d.lm_counter, 1u) == (uint32_t)(G - 1);
  }
  csync();
  if (!cx.last || warp != 0) return true;
  __threadfence();
  float bv = -INFINITY;
  int bi = 0x7fffffff;
#pragma unroll 1
  for (int j0 = lane; j0 < G; j0 += 8 * 32) {
    float v[8];
    int ix[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int j = j0 + 32 * k;
      v[k] = j < G ? __ldcg(d.lm_partial_val + j) : -INFINITY;
      ix[k] = j < G ? __ldcg(d.lm_partial_idx + j) : 0x7fffffff;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (better(v[k], ix[k], bv, bi)) {
        bv = v[k];
        bi = ix[k];
      }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane == 0) head_finish(bi);
  CSTAMP(L, 5);
  return true;
}

// Wait (bounded) until the start gate is nonzero (acquire); false when it
// stayed closed.
__device__ __noinline__ bool gate_open(const int32_t* gate, unsigned long long limit_ns) {
  const unsigned long long t0 = global_ns();
#pragma unroll 1
  while (ld_acquire_gpu(reinterpret_cast<const uint32_t*>(gate)) == 0u)
    if (global_ns() - t0 > limit_ns) return false;
  return true;
}


// After cluster barrier 3 of layer l (producer warp): the routing the
// consumers compute, then the selected experts' gate/up rows of this CTA and,
// once those landed, its down rows -- needed only after the up units and the
// hidden exchange, they would otherwise share the SM's bandwidth with the
// gate/up rows the consumers wait for.
template <bool EP, bool Q8>
__device__ __forceinline__ bool producer_experts(int l, bool ok) {
  const Route rt = route_top2(l);
  int le0, le1;
  local_experts<EP>(rt.sel0, rt.sel1, &le0, &le1);
  if (!ok) return false;
  tma_experts<EP, Q8>(l, le0, le1, false);
  __syncwarp();
  const bool mine = mbar_wait(&bars_s[kFE], (armed_s[kFE] - 1u) & 1u, ps.d.status, lim_s);
  if (!mine) raise_abort();
  if (!__all_sync(0xffffffffu, mine)) return false;
  tma_experts<EP, Q8>(l, le0, le1, true);
  return true;
}

// The producer warp's program: it stages, one layer ahead, everything that
// does not depend on the layer's routing -- the next layer's first K/V chunk,
// out_proj tile, router + norm weights and q/k/v rows, each once the
// consumers have read the region for the last time -- and, right after
// cluster barrier 3, the rows of the experts this layer selected; then the
// LM-head ring.  It arrives at every cluster barrier as soon as it may, so
// the consumers never wait for it; after a failed wait it keeps taking the
// cluster barriers without staging.
template <bool EP, bool Q8>
__device__ __noinline__ void producer(const CStepParams& P, bool att, bool ok) {
  const mie_step_desc& d = ps.d;
  const CGeom& g = ps.g;
  const int L = d.num_layers;
  const Split a = split_of(cx.pos);
  const int n0 = min(g.chunk_tok, a.t1 - a.t0);
  if (ok && att && n0 > 0) tma_kv(0, a.h, a.t0, n0);
#pragma unroll 1
  for (int l = 0; l < L; ++l) {
    if (l + 2 < L && l + 2 >= kLaySlots) layer_fetch(P, l + 2, kProd);  // into the slot of layer l - 2
    if (att) {
      cluster_arrive();  // barrier 1 (q, k_new, v_new)
      cluster_wait();
      cluster_arrive();  // barrier 2 (split results)
      cluster_wait();
      cluster_arrive();  // barrier 3 (x_mid, router partials)
      if (l + 1 < L) {
        ok = pwait(ok, kEK);
        if (ok && n0 > 0) tma_kv(l + 1, a.h, a.t0, n0);
        ok = pwait(ok, kEO);
        if (ok) tma_otile(P, l + 1);
      }
      cluster_wait();
      ok = producer_experts<EP, Q8>(l, ok);
      ok = pwait(ok, kER);
      if (ok) tma_side(l + 1);
      if (l + 1 < L) {
        ok = pwait(ok, kEA);
        if (ok) tma_qkv(l + 1);
      }
    } else {
      cluster_arrive();  // barrier 3 (x_mid, router partials)
      cluster_wait();
      ok = producer_experts<EP, Q8>(l, ok);
      ok = pwait(ok, kER);
      if (ok) tma_side(l + 1);
    }
  }
  // the LM-head ring over regions A..D, free after the last down projection
  ok = pwait(ok, kED);
  if (ok) tma_head(0, g.head_stages);
  int v0, v1;
  split32(d.vocab, blockIdx.x, g.G, &v0, &v1);
  const int nst = (v1 - v0 + g.head_rows - 1) / g.head_rows;
#pragma unroll 1
  for (int i = 0; i + g.head_stages < nst; ++i) {
    ok = pwait(ok, kEH + i % g.head_stages);
    if (ok) tma_head(i + g.head_stages, 1);
  }
}

// EP: expert parallel (ps.g.peer_world > 1); Q8: int8 experts (ps.g.qbits
// 8).  Separate instantiations, so the bf16 single-GPU step carries none of
// their code.
template <bool EP, bool Q8>
__global__ void __launch_bounds__(kT, 1) cstep_kernel(const __grid_constant__ CStepParams P) {
  CSTAMP(P.d.num_layers, 3);
  // under programmatic dependent launch the next step's CTAs may take the SMs
  // this grid's CTAs leave; they stage their first weights, then wait
  pdl_trigger();
  {
    constexpr int kWords = (int)(sizeof(CShared) / 8);
    static_assert(sizeof(mie_step_desc) % 8 == 0 && sizeof(CGeom) % 8 == 0, "8-byte words");
    const int i = threadIdx.x;
    if (i < kWords) {
      const uint64_t* src = i < (int)(sizeof(mie_step_desc) / 8)
                                ? reinterpret_cast<const uint64_t*>(&P.d) + i
                                : reinterpret_cast<const uint64_t*>(&P.g) + (i - (int)(sizeof(mie_step_desc) / 8));
      reinterpret_cast<uint64_t*>(&ps)[i] = *src;
    }
#pragma unroll 1
    for (int l = 0; l < kLaySlots && l < P.d.num_layers; ++l) layer_fetch(P, l, 128 + 16 * l);
    if (threadIdx.x == 0) {
      cx.pos = 0;
#pragma unroll 1
      for (int b = 0; b < kNB; ++b) {
        // full barriers: one arrival per thread of the filling side; empty: one
        // full barriers filled by the consumers' cp.async: one arrival per
        // consumer thread; by the producer's bulk copies, and empty barriers: one
        const bool cons = b == kFK2;
        mbar_init(&bars_s[b], cons ? (uint32_t)kCT : 1u);
        armed_s[b] = done_s[b] = 0;
        if (b < kNF)
          for (int w = 0; w < kCW; ++w) wdone_s[w][b] = 0;
      }
      fence_barrier_init();
    }
    __syncthreads();
  }
  const mie_step_desc& d = ps.d;
  const bool att = (int)(blockIdx.x / kCS) < d.num_heads;
  // layer 0's q/k/v rows, out_proj tile, router and norm weights depend on the
  // CTA alone: the producer warp stages them before the wait
  if (threadIdx.x >= kProd) {
    if (att) {
      tma_qkv(0);
      tma_otile(P, 0);
    }
    tma_side(0);
  }
  // the previous step's writes are visible from here on
  pdl_wait();
  bool ok = true;
  if (threadIdx.x == 0) {
    const int done_v = d.done ? __ldcg(d.done) : 0;
    const int lc = d.log_count ? __ldcg(d.log_count) : 0;
    const int lim = d.step_limit ? __ldcg(d.step_limit) : 0;
    const uint64_t hstep = ll_ld(ps.g.ll + kHdrStep);
    const int p = __ldcg(d.pos);
    const int64_t t = __ldcg(d.token);
    int stop = done_v || (d.step_limit && d.log_count && lc >= lim);
    lim_s = d.wait_limit_ns > 0 ? (unsigned long long)d.wait_limit_ns : kWaitLimitNs;
    cx.step = (uint32_t)hstep + 1u;
    cx.pstep = EP ? *reinterpret_cast<volatile const uint32_t*>(ps.g.peer_seq) + 1u : 0u;
    cx.log_k = lc;
    if (!stop && (p < 0 || p >= d.max_pos || t < 0 || t >= d.vocab)) {
      if (blockIdx.x == 0) set_status(d.status, MIE_ERR_RANGE);
      stop = 1;
    }
    int64_t blk = stop ? 0 : p / d.block_size;
    if (!stop && d.block_table) {
      const int pb = __ldcg(d.block_table + blk);
      if (pb < 0 || pb >= d.num_blocks) {
        if (blockIdx.x == 0) set_status(d.status, MIE_ERR_RANGE);
        stop = 1;
      }
      blk = pb;
    }
    cx.pos = p;
    cx.tok = t;
    cx.slot = stop ? 0 : blk * d.kv_stride_block + (int64_t)(p % d.block_size) * d.kv_stride_tok;
    cx.blk0 = 0;
    if (!stop) {
      int t0, t1;
      split32(p, (int)(blockIdx.x % kCS), kCS, &t0, &t1);
      cx.blk0 = t0 / d.block_size;
    }
    cx.stop = stop;
  } else if (d.block_table && threadIdx.x <= kBlkCache) {
    // physical block ids of this split's old tokens, the same for every layer
    const int p = __ldcg(d.pos), i = threadIdx.x - 1;
    if (p >= 0 && p < d.max_pos) {
      int t0, t1;
      split32(p, (int)(blockIdx.x % kCS), kCS, &t0, &t1);
      const int b0 = t0 / d.block_size;
      if (t1 > t0 && b0 + i <= (t1 - 1) / d.block_size) blk_s[i] = __ldcg(d.block_table + b0 + i);
    }
  }
  __syncthreads();
  // the stop decision reads the same device state in every CTA: grid-uniform
  if (cx.stop) {
    drain_copies();
    return;
  }
  // a closed start gate ends this CTA's part of the step; it still takes every
  // cluster barrier
  if (d.start_gate) {
    __shared__ int gate_ok;
    if (threadIdx.x == 0) {
      gate_ok = gate_open(d.start_gate, lim_s) ? 1 : 0;
      if (!gate_ok) set_status(d.status, MIE_ERR_TIMEOUT);
    }
    __syncthreads();
    ok = gate_ok != 0;
  }
  CSTAMP(d.num_layers, 4);
  if (threadIdx.x >= kProd) {
    producer<EP, Q8>(P, att, ok);
  } else {
#pragma unroll 1
    for (int l = 0; l < d.num_layers; ++l) {
      if (att) ok = att_phase<EP>(P, l, ok);
      ok = moe_phase<EP, Q8>(P, l, ok, att);
    }
    head_phase<EP>(ok);
  }
  drain_copies();
}

// ---- host side ----
std::mutex g_cluster_mutex;
int g_max_clusters[64] = {0};  // per device: clusters of the kernel that fit at once (0: not queried)

}  // namespace

int cstep_geometry(const mie_step_desc& d, CGeom* out) {
  if (d.step_kernel == MIE_STEP_FLAT) return MIE_ERR_UNSUPPORTED;
  if (d.dtype != MIE_BF16 || d.kv_dtype != MIE_BF16) return MIE_ERR_UNSUPPORTED;
  if (d.norm != MIE_NORM_RMS || d.act != MIE_ACT_SWIGLU || d.top_k != 2) return MIE_ERR_UNSUPPORTED;
  if (d.head_dim != kHd || d.num_heads * kHd != d.hidden_dim) return MIE_ERR_UNSUPPORTED;
  const int D = d.hidden_dim, Hx = d.expert_hidden_dim, E = d.num_experts, H = d.num_heads;
  if (D > 768 || D % kPV || Hx > 768 || Hx % kPV || Hx <= 0 || E < 2 || E > 32) return MIE_ERR_UNSUPPORTED;
  if (d.num_layers <= 0 || d.num_layers > kMaxStepLayers) return MIE_ERR_UNSUPPORTED;
  if (!d.rope_cos || !d.rope_sin || d.pos_embedding || d.lm_bias || d.final_norm_b) return MIE_ERR_UNSUPPORTED;
  if (d.sample_temperature > 0.f) return MIE_ERR_UNSUPPORTED;  // the device sampler runs on the flat step
  // expert parallel: the ranks' partials travel inside the step (moe_peer),
  // never through moe_partial
  const mie_peer_reduce_args* pr = d.moe_peer;
  const bool ep = pr && pr->world > 1;
  if (d.moe_partial) return MIE_ERR_UNSUPPORTED;
  if (ep) {
    if (pr->world > MIE_PEER_MAX_RANKS || pr->rank < 0 || pr->rank >= pr->world || pr->n != D || !pr->seq)
      return MIE_ERR_INVALID;
    for (int r = 0; r < pr->world; ++r)
      if (!pr->bufs[r] || reinterpret_cast<uintptr_t>(pr->bufs[r]) % 8) return MIE_ERR_INVALID;
    if (d.expert_count <= 0 || d.expert_base < 0 || d.expert_base + d.expert_count > E) return MIE_ERR_INVALID;
  } else if ((d.expert_count && d.expert_count != E) || d.expert_base) {
    return MIE_ERR_UNSUPPORTED;
  }
  // int8 experts: groups of a power of two >= 32 along rows of 16-byte
  // multiples; int4, or int8 with expert parallelism, run layer by layer
  int qgsh = 0;
  if (d.expert_bits) {
    const int gs = d.group_size;
    if (d.expert_bits != 8 || ep) return MIE_ERR_UNSUPPORTED;
    if (gs < 32 || (gs & (gs - 1)) || D % gs || Hx % gs || D % 16 || Hx % 16) return MIE_ERR_UNSUPPORTED;
    while ((1 << qgsh) < gs) ++qgsh;
    for (int l = 0; l < d.num_layers; ++l) {
      const mie_layer_desc& y = d.layers[l];
      if (!y.w1_scale || !y.w3_scale || !y.w2_scale) return MIE_ERR_INVALID;
      if ((reinterpret_cast<uintptr_t>(y.w1) | reinterpret_cast<uintptr_t>(y.w3) | reinterpret_cast<uintptr_t>(y.w2)) & 15u)
        return MIE_ERR_INVALID;
    }
  }
  if (d.kv_stride_tok != kHd || (d.kv_stride_block * 2) % 16 || (d.kv_stride_head * 2) % 16)
    return MIE_ERR_UNSUPPORTED;
  for (int l = 0; l < d.num_layers; ++l) {
    const mie_layer_desc& y = d.layers[l];
    if (y.qkv_b || y.out_b || y.b1 || y.b2 || y.attn_norm_b || y.moe_norm_b || !y.w3) return MIE_ERR_UNSUPPORTED;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MIE_ERR_CUDA;
  CGeom& g = *out;
  g = CGeom{};
  // shared memory layout
  const uint32_t rbD = (uint32_t)D * 2u, rbH = (uint32_t)Hx * 2u;
  g.np_max = (kHd / 2 + kCS - 1) / kCS;
  g.nv_max = (kHd + kCS - 1) / kCS;
  g.orows = (D + kCS - 1) / kCS;
  g.chunk_tok = 256;
  uint32_t so = 0;
  auto stake = [&](uint32_t bytes) {
    so = (so + 127) & ~127u;
    const uint32_t at = so;
    so += bytes;
    return at;
  };
  // the grid size decides the expert shares; start from the cached cluster count
  int nc;
  {
    std::lock_guard<std::mutex> lock(g_cluster_mutex);
    nc = g_max_clusters[dev];
  }
  if (nc <= 0) return MIE_ERR_UNSUPPORTED;  // cstep_set_attributes found no room for the kernel
  if (nc > 40) nc = 40;
  if (nc < H) return MIE_ERR_UNSUPPORTED;  // one cluster per head
  g.NC = nc;
  g.G = nc * kCS;
  if ((int64_t)d.vocab * g.G >= (1ll << 32) || (int64_t)d.max_pos * kCS >= (1ll << 32)) return MIE_ERR_UNSUPPORTED;
  if (d.lm_grid < g.G) return MIE_ERR_INVALID;
  g.nu_max = (2 * Hx + g.G - 1) / g.G;
  g.nr_max = (D + g.G - 1) / g.G;
  // per-thread epilogues: one up unit / out_proj row / down row per consumer thread
  if (2 * g.nu_max > kCT || g.orows > kCT || g.nr_max > kCT) return MIE_ERR_UNSUPPORTED;
  if (2 * g.nr_max > kCW) return MIE_ERR_UNSUPPORTED;  // the down GEMV: one row per consumer warp
  const uint32_t a_bytes = (uint32_t)max(4 * g.np_max + g.nv_max, 2 * g.nu_max) * rbD;
  // everything the LM head does not use comes first: after the last layer it
  // is one contiguous ring of LM-head stages
  g.sm_k = stake((uint32_t)(2 * g.chunk_tok * kHd * 2));
  g.sm_o = stake((uint32_t)(g.orows * kHd * 2));
  g.sm_a = stake(a_bytes);
  g.sm_d = stake(2u * (uint32_t)g.nr_max * rbH);
  g.sm_r = stake((uint32_t)(E + 2) * rbD);
  g.sm_xm = stake(8u * D);
  g.sm_g = stake(2u * 3u * kHd * 4u);
  g.sm_mg = stake(2u * kCS * kMg * 4u);
  g.sm_qkv = stake((uint32_t)(4 * g.np_max + g.nv_max) * 4u);
  g.sm_sc = stake((uint32_t)g.chunk_tok * 4u);
  g.sm_h = stake(8u * Hx);
  g.sm_pr = stake((uint32_t)(H + 1) * g.orows * 4u);
  g.sm_ov = stake((kHd + 4) * 4u);
  // the LM head's vectors and the final norm weights after the ring
  const uint32_t tail = 4u * D * 2u + 2u * D + 4u * (uint32_t)max(kT, max(E, 2 * g.nu_max)) + 8u * kCS +
                        8u * kCS * (uint32_t)E + 6u * 128u;
  if (so + tail > kStepMaxSmem) return MIE_ERR_UNSUPPORTED;
  so = kStepMaxSmem - tail;  // the ring takes whatever shared memory is left
  g.sm_fn = stake(2u * D);
  g.sm_x = stake(4u * D);
  g.sm_xn = stake(4u * D);
  g.sm_ab = stake(4u * (uint32_t)max(kT, max(E, 2 * g.nu_max)));
  g.sm_ss = stake(8u * kCS);
  g.sm_rp = stake(8u * kCS * (uint32_t)E);
  g.smem = (so + 127) & ~127u;
  if (g.smem > kStepMaxSmem) return MIE_ERR_UNSUPPORTED;
  // LM-head ring over [sm_k, sm_fn): stages of four rows per consumer warp
  g.head_rows = 4 * kCW;
  const uint32_t ring = g.sm_fn - g.sm_k;
  g.head_stages = (int)(ring / ((uint32_t)g.head_rows * rbD));
  if (g.head_stages > kStepHeadStagesMax) g.head_stages = kStepHeadStagesMax;
  if (g.head_stages < 2) return MIE_ERR_UNSUPPORTED;
  // exchange words, two copies each
  int64_t off = 8;
  auto take = [&](int64_t words) {
    const int64_t at = off;
    off += (words + 1) & ~int64_t(1);
    return at;
  };
  for (int p = 0; p < 2; ++p) {
    g.off_x[p] = take(D);
    g.off_p[p] = take((int64_t)H * D);
    g.off_h[p] = take(2 * (int64_t)Hx);
  }
  g.words = off;
  if (d.expert_bits) {
    // int8 rows first, their scales after them, inside regions A and D
    g.qbits = 8;
    g.qgsh = qgsh;
    g.q_a_scale = ((uint32_t)(2 * g.nu_max * D) + 15u) & ~15u;
    g.q_d_scale = ((uint32_t)(2 * g.nr_max * Hx) + 15u) & ~15u;
    if (g.q_a_scale + (uint32_t)(2 * g.nu_max * (D >> qgsh)) * 4u > a_bytes ||
        g.q_d_scale + (uint32_t)(2 * g.nr_max * (Hx >> qgsh)) * 4u > 2u * (uint32_t)g.nr_max * rbH)
      return MIE_ERR_UNSUPPORTED;
  }
  g.peer_world = 1;
  if (ep) {
    g.peer_rank = pr->rank;
    g.peer_world = pr->world;
    for (int r = 0; r < pr->world; ++r) g.peer_bufs[r] = pr->bufs[r];
    g.peer_seq = pr->seq;
  }
  return MIE_OK;
}

int cstep_launch(const mie_step_desc& d, const CGeom& g, uint64_t* scratch, cudaStream_t st) {
  static CStepParams p;  // large: not on the stack (launches are made from one host thread at a time)
  static std::mutex m;
  std::lock_guard<std::mutex> lock(m);
  p.d = d;
  p.g = g;
  p.g.ll = scratch;
  EncodeTiledFn fn = encode_fn();
  if (!fn) return MIE_ERR_CUDA;
  const int D = d.hidden_dim;
  for (int l = 0; l < d.num_layers; ++l) {
    p.layers[l] = d.layers[l];
    // out_proj [D rows, D columns] bf16; a tile = hd columns (one head) x orows rows
    const cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)D};
    const cuuint64_t strides[1] = {(cuuint64_t)D * 2u};
    const cuuint32_t box[2] = {(cuuint32_t)kHd, (cuuint32_t)g.orows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(&p.omap[l], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(d.layers[l].out_w), dims,
                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return MIE_ERR_INVALID;
  }
  p.d.layers = nullptr;
#ifdef MIE_STEP_STAMPS
  if (d.num_layers + 1 > kStampLayers || g.G > 160) return MIE_ERR_UNSUPPORTED;
#endif
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)g.G);
  cfg.blockDim = dim3(kT);
  cfg.dynamicSmemBytes = g.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kCS;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = d.use_pdl ? 2 : 1;
  const cudaError_t e = cudaLaunchKernelEx(
      &cfg, g.peer_world > 1 ? cstep_kernel<true, false> : g.qbits ? cstep_kernel<false, true> : cstep_kernel<false, false>,
      p);
  if (e != cudaSuccess) {
    note_cuda_error(e, "cudaLaunchKernelEx(cluster step)");
    return MIE_ERR_CUDA;
  }
  return MIE_OK;
}

// Once per device (from mie_init): the shared-memory attribute, then how many
// clusters of the kernel the device holds at once with its largest shared
// memory footprint.
void cstep_set_attributes() {
  set_max_smem(cstep_kernel<false, false>);
  set_max_smem(cstep_kernel<true, false>);
  set_max_smem(cstep_kernel<false, true>);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kCS * 8);
  cfg.blockDim = dim3(kT);
  cfg.dynamicSmemBytes = kStepMaxSmem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kCS;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // every instantiation must fit the grid: the smallest count
  int n = 0, n_ep = 0, n_q8 = 0;
  cudaError_t e = cudaOccupancyMaxActiveClusters(&n, cstep_kernel<false, false>, &cfg);
  if (e == cudaSuccess) e = cudaOccupancyMaxActiveClusters(&n_ep, cstep_kernel<true, false>, &cfg);
  if (e == cudaSuccess) e = cudaOccupancyMaxActiveClusters(&n_q8, cstep_kernel<false, true>, &cfg);
  if (e != cudaSuccess) {
    note_cuda_error(e, "cudaOccupancyMaxActiveClusters(cluster step)");
    n = 0;
  }
  n = min(n, min(n_ep, n_q8));
  std::lock_guard<std::mutex> lock(g_cluster_mutex);
  g_max_clusters[dev] = n;
}

#ifdef MIE_STEP_STAMPS
extern "C" int mie_debug_cstep_stamps(unsigned long long* host, int64_t count) {
  return cudaMemcpyFromSymbol(host, g_cstep_stamps, sizeof(unsigned long long) * (size_t)count) == cudaSuccess
             ? MIE_OK
             : MIE_ERR_CUDA;
}
#endif

}  // namespace mie
