// Persistent decode step: the whole batch-one decode step (all layers + LM
// head) in ONE launch of one CTA per SM, sm_100a.
//
// The per-op launch sequence (qkv -> attention -> out_proj -> MoE per layer,
// LM head at the end; src/moe_engine/model.py:543-565 of the reference) pays a
// launch, a prologue and a grid-wide drain per kernel.  Here every CTA walks
// the same program of phases and the phases hand their results to each other
// through small "LL" exchanges in global memory: every value travels as one
// 64-bit word {f32 value, u32 tag} written with a single 64-bit store, and a
// consumer polls the words it needs until their tag equals the tag of the
// current (step, layer).  A word is complete the moment its tag is visible, so
// no fence, counter or grid barrier is needed.
//
// Phases of layer l (G CTAs; the first H*S CTAs are attention CTAs, CTA
// (h, s) = split s of head h):
//
//   ATT    every CTA: x (exchange A, or the token embedding for l = 0) ->
//          norm.  Attention CTAs compute q_h (all hd rows of head h) locally,
//          plus their share of the new token's k (RoPE pairs) and v rows,
//          which they store into the cache slot of the position.  Online
//          softmax over the split's share of the OLD tokens, and the split's
//          share of q.k_new.  -> exchange B: (m, l, q.k_new part, acc).
//   MERGE  attention CTAs: the S entries of their head -> log-sum-exp merge
//          with the new token as one more term -> o_h for their v dims ->
//          exchange C.
//   PROJ   every CTA: its rows of out_proj + bias + residual -> exchange D
//          (x_mid).
//   UP     every CTA: x_mid -> norm -> router -> top-2 (ties to the lower id)
//          -> 2-way softmax -> its up units (gate [+ up] rows) of the two
//          selected experts: h = act(...) -> exchange E.
//   DOWN   every CTA: its output rows: x_mid + sum_k w_k (W2_k h_k + b2_k) ->
//          exchange A of layer l + 1.
//
// Then HEAD: x_L -> final norm -> tied LM head rows -> per-CTA argmax -> the
// last CTA to arrive reduces the CTA results and does the step's device
// bookkeeping (next token, position + 1, token log, EOS flag, step counter).
//
// Weights and old K/V never travel through registers ahead of time: they are
// staged in shared memory by bulk copies (cp.async.bulk, completion counted on
// an mbarrier) issued long before they are needed -- layer l + 1's attention
// inputs right after layer l's attention, layer l + 1's out_proj rows, router
// rows and norm weights right after layer l's down projection, the selected
// experts' rows right after routing, the LM-head rows through a ring.  Every
// GEMV then runs from shared memory.
//
// The code is organised for the instruction cache: one decode step runs every
// phase of every layer, so the code of one layer should stay resident.  The
// phases are thin sequences of calls to a few shared routines (exchange
// receive, norm, GEMV over staged rows, attention core), and loops that need
// no unrolling are not unrolled.
//
// Exchange buffers are reused every second layer (A, B, C, D, E each have two
// copies, by layer parity).  A CTA writes a buffer of layer l + 2 only after it
// consumed exchange D of layer l + 1, to which every CTA contributed after it
// finished reading layer l's copy, so a copy is never overwritten while read.
// Every wait is bounded (kWaitLimitNs); a CTA that gives up records
// MIE_ERR_TIMEOUT, raises the abort word so the others stop waiting, waits
// (bounded) for its own bulk copies still in flight, and leaves.  After that
// the host must zero the scratch before the next step.
//
// Every reduction has a fixed order: results are bit-reproducible run to run.
#include "exchange.cuh"
#include "kernels.h"
#include "stream.cuh"

namespace mie {

namespace {

constexpr int kST = kStepThreads;
constexpr int kSW = kST / 32;

// scratch header words
constexpr int kHdrStep = 0;   // completed steps (the step counter)
constexpr int kHdrAbort = 1;  // nonzero: a CTA gave up waiting

#ifdef MIE_STEP_STAMPS
// Phase timestamps for performance analysis builds only: [CTA][layer][point].
constexpr int kStampLayers = kMaxStepLayers + 1, kStampPoints = 32;
__device__ unsigned long long g_step_stamps[160 * kStampLayers * kStampPoints];
#define STEP_STAMP(l, k) \
  do { \
    if (threadIdx.x == 0) g_step_stamps[(blockIdx.x * kStampLayers + (l)) * kStampPoints + (k)] = global_ns(); \
  } while (0)
#define STEP_STAMP_T(l, k, t) \
  do { \
    if (threadIdx.x == (t)) g_step_stamps[(blockIdx.x * kStampLayers + (l)) * kStampPoints + (k)] = global_ns(); \
  } while (0)
#else
#define STEP_STAMP_T(l, k, t) \
  do { \
  } while (0)
#define STEP_STAMP(l, k) \
  do { \
  } while (0)
#endif

// Limit of every wait of this step (ns), set in the step prologue.
__shared__ unsigned long long wait_ns_s;

// ---------------------------------------------------------------------------
// Exchange words
// ---------------------------------------------------------------------------
// Slow path of a wait, every 64 polls: true when another CTA raised the abort
// word or this wait has run for kWaitLimitNs (then MIE_ERR_TIMEOUT is
// recorded and the abort word raised).
__device__ __noinline__ bool ll_give_up(uint64_t* hdr, int32_t* status, unsigned long long* t0) {
  if (ll_ld(hdr + kHdrAbort)) return true;
  const unsigned long long t = global_ns();
  if (!*t0) {
    *t0 = t;
    return false;
  }
  if (t - *t0 <= wait_ns_s) return false;
  set_status(status, MIE_ERR_TIMEOUT);
  atomicExch(reinterpret_cast<unsigned long long*>(hdr + kHdrAbort), 1ull);
  return true;
}

// The polling part of recv, without the closing barrier: 1 when a wait gave
// up.  With s2 set, *s2 = sum of squares of this thread's words in index
// order (t, t + NT, ...), the order a strided loop over dst would use.  Run
// by threads [0, NT).
template <int NT = kST>
__device__ __forceinline__ int recv_poll(const uint64_t* buf, int n, uint32_t tag, float* dst, const int* gather,
                                         uint64_t* hdr, int32_t* status, float* s2) {
  float acc = 0.f;
#pragma unroll 1
  for (int i0 = threadIdx.x; i0 < n; i0 += NT * 4) {
    uint64_t w[4];
    int at[4];
    unsigned need = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = i0 + NT * j;
      at[j] = i < n ? (gather ? gather[i] : i) : 0;
      if (i < n) {
        w[j] = ll_ld(buf + at[j]);
        need |= 1u << j;
      }
    }
    const unsigned all = need;
    unsigned long long t0 = 0;
#pragma unroll 1
    for (int it = 1;; ++it) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if ((need >> j & 1u) && ll_tag(w[j]) == tag) {
          dst[i0 + NT * j] = ll_val(w[j]);
          need &= ~(1u << j);
        }
      }
      if (!need) break;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (need >> j & 1u) w[j] = ll_ld(buf + at[j]);
      if ((it & 63) == 0 && ll_give_up(hdr, status, &t0)) return 1;
    }
    if (s2) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (all >> j & 1u) {
          const float v = ll_val(w[j]);
          acc = fmaf(v, v, acc);
        }
    }
  }
  if (s2) *s2 = acc;
  return 0;
}

// Receive n exchange words: dst[i] = value of buf[idx(i)] (idx(i) = i when
// gather is null, else gather[i]) once its tag equals `tag`.  Thread t owns
// words t, t + kST, ...; all of its pending words are polled again together,
// so a thread sees its last word one load round trip after it landed.  Called
// by every thread; true for all of them, or false for all when a wait gave up.
__device__ __noinline__ bool recv(const uint64_t* buf, int n, uint32_t tag, float* dst, const int* gather,
                                  uint64_t* hdr, int32_t* status) {
  return __syncthreads_or(recv_poll(buf, n, tag, dst, gather, hdr, status, nullptr)) == 0;
}

// ---------------------------------------------------------------------------
// Small helpers
// ---------------------------------------------------------------------------
// Contiguous share of `total` items for CTA `c` of `g` in 32-bit arithmetic
// (total * g < 2^32, checked on the host).
__device__ __forceinline__ void split32(int total, int c, int g, int* begin, int* end) {
  *begin = (int)(((uint32_t)total * (uint32_t)c) / (uint32_t)g);
  *end = (int)(((uint32_t)total * (uint32_t)(c + 1)) / (uint32_t)g);
}
// Typed element load (the step kernel knows its weight type at compile time).
template <typename T>
__device__ __forceinline__ float ldw(const void* p, int64_t i) {
  return Elem<T>::to_f(static_cast<const T*>(p)[i]);
}
__device__ __forceinline__ const uint4* rowp(const void* base, int64_t row, int64_t row_bytes) {
  return reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(base) + row * row_bytes);
}
__device__ __forceinline__ float gelu_erf(float v) { return 0.5f * v * (1.0f + erff(v * 0.7071067811865476f)); }
__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

// ---------------------------------------------------------------------------
// Per-step state shared by the phases (shared memory of each CTA).
// ---------------------------------------------------------------------------
struct StepCtx {
  int pos;        // position of the input token
  int stop;       // nonzero: skip the step (EOS reached or bad input)
  uint32_t step;  // this step's number (tags)
  int64_t tok;    // input token
  int64_t slot;   // cache offset (elements) of the new token's slot, head 0
  float m, l;     // attention: running max and normaliser of this split
  int last;       // this CTA finished the LM head last
  int blk0;       // first cache block of this CTA's old tokens (blk_s[0])
  int log_k;      // *log_count at the start of the step
};
constexpr int kStepBlkCache = 64;  // block ids of a split cached per step
__shared__ StepCtx cx_s;
// The launch parameters the phases read, copied to shared memory at the
// start (a read of a kernel parameter through a reference costs ~250 cycles,
// a shared-memory read ~30): the step descriptor, the geometry and a window
// of kLayerSlots layer descriptors -- layer l in slot l % kLayerSlots; the
// descriptor of layer l + 2 is copied during layer l.
struct StepShared {
  mie_step_desc d;
  StepGeom g;
};
constexpr int kLayerSlots = 4;
__shared__ StepShared ps_s;
__shared__ mie_layer_desc lay_s[kLayerSlots];
__device__ __forceinline__ const mie_layer_desc& layer_at(int l) { return lay_s[l & (kLayerSlots - 1)]; }
// Copy layer l's descriptor into its slot (threads [first, first + 16)).
__device__ __forceinline__ void layer_fetch(const StepParams& P, int l, int first) {
  constexpr int kWords = (int)(sizeof(mie_layer_desc) / 8);
  const int i = (int)threadIdx.x - first;
  if (i >= 0 && i < kWords)
    reinterpret_cast<uint64_t*>(&lay_s[l & (kLayerSlots - 1)])[i] =
        reinterpret_cast<const uint64_t*>(&P.layers[l])[i];
}
__shared__ float red_s[kSW];
__shared__ float red2_s[kSW];  // the attention core's sum (its max uses red_s): one barrier each
__shared__ int gat_s[kST];  // merge: exchange word index of each received value
__shared__ int blk_s[kStepBlkCache];  // physical block ids of this CTA's old tokens
__shared__ float bestv_s[kSW];
__shared__ int besti_s[kSW];

// ---------------------------------------------------------------------------
// Device sampler (temperature > 0).  Gumbel-max: argmax_i (l_i / T + G_i) with
// G_i = -log(-log U_i) draws i with probability softmax(l / T)_i; U_i comes
// from the SplitMix64 finaliser (Steele, Lea, Flood 2014) of (seed, position,
// token id), so a step's draw is reproducible and independent of the grid.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float gumbel(uint64_t seed, int pos, int row) {
  uint64_t z = seed + 0x9E3779B97F4A7C15ull * (((uint64_t)(uint32_t)pos << 32) + (uint64_t)(uint32_t)row + 1u);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  const float u = ((float)(z >> 40) + 0.5f) * (1.0f / 16777216.0f);  // (0, 1)
  return -logf(-logf(u));
}
// Sort key of (logit, token): descending key order = larger logit first, then
// lower token id; 0 sorts below every real logit.
__device__ __forceinline__ uint64_t logit_key(float v, int row) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((uint64_t)b << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)row);
}
__device__ __forceinline__ float key_logit(uint64_t k) {
  uint32_t b = (uint32_t)(k >> 32);
  b = (b & 0x80000000u) ? (b & 0x7FFFFFFFu) : ~b;
  return __uint_as_float(b);
}
__device__ __forceinline__ int key_row(uint64_t k) { return (int)(0xFFFFFFFFu - (uint32_t)k); }
// Descending bitonic sort of keys[0, n) in shared memory (n a power of two),
// by the whole CTA; ends with a barrier.
__device__ __noinline__ void sort_keys_desc(uint64_t* keys, int n) {
  __syncthreads();
#pragma unroll 1
  for (int size = 2; size <= n; size <<= 1) {
#pragma unroll 1
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
#pragma unroll 1
      for (int t = threadIdx.x; t < n / 2; t += kST) {
        const int i = 2 * t - (t & (stride - 1)), j = i + stride;  // pair (i, j), i has bit `stride` clear
        const bool desc = (i & size) == 0;
        const uint64_t a = keys[i], b = keys[j];
        if ((a < b) == desc) {
          keys[i] = b;
          keys[j] = a;
        }
      }
      __syncthreads();
    }
  }
}
// mbarriers of the bulk-copy staging, with per-barrier counts of armed and
// completed phases (a wait uses parity = completed & 1).
constexpr int kBarAtt = 0, kBarKv = 1, kBarSide = 2, kBarMoe = 3, kBarDown = 4, kBarHead = 5;
constexpr int kNumBars = kBarHead + kStepHeadStagesMax;
__shared__ __align__(8) uint64_t bars_s[kNumBars];
__shared__ uint32_t bar_armed_s[kNumBars], bar_done_s[kNumBars];
extern __shared__ __align__(128) uint8_t sm[];

__device__ __forceinline__ uint32_t tag_of(int l) { return (cx_s.step << 8) | (uint32_t)l; }
template <typename T>
__device__ __forceinline__ T* smem_at(uint32_t off) {
  return reinterpret_cast<T*>(sm + off);
}

// ---------------------------------------------------------------------------
// Bulk-copy staging
// ---------------------------------------------------------------------------
// Arm barrier b for `bytes` of bulk copies (one thread, before its copies).
__device__ __forceinline__ void bar_arm(int b, uint32_t bytes) {
  bar_armed_s[b] += 1;
  mbar_arrive_expect_tx(&bars_s[b], bytes);
}
// Bulk copy global -> shared counted on barrier b (16-byte aligned, size a
// multiple of 16), in pieces of at most 64 KB.  Everything a step streams
// once (layer weights, K/V) is marked evict-first in L2; `keep` (the tied LM
// head, 77 MB for the miniMoE vocabulary) is marked evict-last, so it can
// stay in the 126 MB L2 from one decode step to the next.
__device__ __noinline__ void bulk_copy(void* dst, const void* src, uint32_t bytes, int b, bool keep = false) {
  const uint64_t pol = keep ? policy_evict_last() : policy_evict_first();
#pragma unroll 1
  for (uint32_t o = 0; o < bytes; o += 65536u)
    bulk_g2s_stream(static_cast<uint8_t*>(dst) + o, static_cast<const uint8_t*>(src) + o, min(65536u, bytes - o),
                    &bars_s[b], pol);
}
// Every thread: wait for the oldest armed phase of barrier b (bounded).
__device__ __noinline__ bool bar_wait(int b, uint64_t* hdr, int32_t* status) {
  const bool ok = mbar_wait(&bars_s[b], bar_done_s[b] & 1u, status, wait_ns_s);
  if (!ok) atomicExch(reinterpret_cast<unsigned long long*>(hdr + kHdrAbort), 1ull);
  const int bad = __syncthreads_or(!ok);
  if (threadIdx.x == 0) bar_done_s[b] += 1;
  return !bad;
}
// PROJ runs on threads [0, kProjThreads): the last two warps issue the next
// layer's bulk copies meanwhile, which can take microseconds when the copy
// engine is busy, and join at the phase's closing barrier.
constexpr int kProjThreads = kST - 64;
// Threads [0, kProjThreads): receive n exchange words into dst and wait
// (bounded) for the copies of barrier b; one named barrier (id 1) over those
// threads closes both.  True for all of them, or false for all when a wait
// gave up.
__device__ __noinline__ bool recv_part(const uint64_t* buf, int n, uint32_t tag, float* dst, int b, uint64_t* hdr,
                                       int32_t* status) {
  int bad = recv_poll<kProjThreads>(buf, n, tag, dst, nullptr, hdr, status, nullptr);
  bool waited = false;
  if (!bad) {
    waited = mbar_wait(&bars_s[b], bar_done_s[b] & 1u, status, wait_ns_s);
    if (!waited) {
      atomicExch(reinterpret_cast<unsigned long long*>(hdr + kHdrAbort), 1ull);
      bad = 1;
    }
  }
  uint32_t any;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbarrier.red.or.pred p, 1, %2, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(any)
      : "r"(bad), "n"(kProjThreads)
      : "memory");
  if (any) return false;
  if (waited && threadIdx.x == 0) bar_done_s[b] += 1;
  return true;
}
// Barrier over threads [0, kProjThreads) (named barrier 1).
__device__ __forceinline__ void bar_sync_part() {
  asm volatile("bar.sync 1, %0;" ::"n"(kProjThreads) : "memory");
}
// Before leaving early: wait (bounded) for every armed copy not waited for,
// so no bulk copy lands in shared memory after the CTA left.
__device__ __noinline__ void drain_copies() {
  if (threadIdx.x != 0) return;
#pragma unroll 1
  for (int b = 0; b < kNumBars; ++b)
    while (bar_done_s[b] < bar_armed_s[b]) {
      mbar_wait(&bars_s[b], bar_done_s[b] & 1u, nullptr);
      bar_done_s[b] += 1;
    }
}

// Work split of the attention CTAs (CTA (h, s) = split s of head h).
struct AttSplit {
  bool att;
  int h, s, p0, nkp, v0, nvd, t0, t1;
};
__device__ __forceinline__ AttSplit att_split(const StepGeom& g, int hd, int pos) {
  AttSplit a;
  const int c = blockIdx.x, S = g.S;
  a.att = c < g.natt;
  a.h = a.att ? c / S : 0;
  a.s = a.att ? c % S : 0;
  int p1, v1;
  split32(hd / 2, a.s, S, &a.p0, &p1);  // k RoPE pairs
  split32(hd, a.s, S, &a.v0, &v1);      // v rows / output dims
  split32(pos, a.s, S, &a.t0, &a.t1);   // old tokens
  a.nkp = a.att ? p1 - a.p0 : 0;
  a.nvd = a.att ? v1 - a.v0 : 0;
  if (!a.att) a.t0 = a.t1 = 0;
  return a;
}

// K/V of tokens [ta, ta + n) of head h -> shared memory (K then V), counted
// on barrier b.  One warp calls this; its lane 0 arms, the lanes issue one
// copy per (block, K or V) segment.  Block ids of this CTA's first
// kStepBlkCache blocks come from the per-step copy in shared memory.
template <typename KV>
__device__ __noinline__ void kv_issue(const mie_step_desc& d, const StepGeom& g, const mie_layer_desc& ly, int h,
                                      int ta, int n, int b) {
  const int lane = threadIdx.x & 31, hd = d.head_dim, bs = d.block_size;
  if (lane == 0) bar_arm(b, (uint32_t)(2 * n * hd * sizeof(KV)));
  __syncwarp();
  KV* dst = smem_at<KV>(g.sm_kv);
  const int b0 = ta / bs, b1 = (ta + n - 1) / bs;
#pragma unroll 1
  for (int bi = b0 + lane; bi <= b1; bi += 32) {
    const int tb = max(ta, bi * bs), te = min(ta + n, (bi + 1) * bs);
    int64_t blk = bi;
    if (d.block_table) {
      const int k = bi - cx_s.blk0;
      const int pb = (k >= 0 && k < kStepBlkCache) ? blk_s[k] : __ldg(d.block_table + bi);
      if (pb < 0 || pb >= d.num_blocks) set_status(d.status, MIE_ERR_RANGE);
      blk = (pb < 0 || pb >= d.num_blocks) ? 0 : pb;
    }
    const int64_t off = blk * d.kv_stride_block + (int64_t)h * d.kv_stride_head + (int64_t)(tb % bs) * d.kv_stride_tok;
    const uint32_t bytes = (uint32_t)((te - tb) * hd * sizeof(KV));
    bulk_copy(dst + (size_t)(tb - ta) * hd, static_cast<const KV*>(ly.k_cache) + off, bytes, b);
    bulk_copy(dst + (size_t)g.chunk_tok * hd + (size_t)(tb - ta) * hd, static_cast<const KV*>(ly.v_cache) + off,
              bytes, b);
  }
}

// Norm weight (and bias) of D elements -> shared memory (one thread).
__device__ __forceinline__ void norm_copy(void* dst, const void* w, const void* b, uint32_t rb, int bar) {
  bulk_copy(dst, w, rb, bar);
  if (b) bulk_copy(static_cast<uint8_t*>(dst) + rb, b, rb, bar);
}

// Stage layer l's attention weights (whole calling warp: lane 0 arms the
// barrier, lanes 0-4 issue one copy each): the attention norm weights; for
// attention CTAs also q rows [0, q_stage) of the head and this CTA's k / v
// rows (k pair first halves, second halves, v rows).
template <typename W>
__device__ __noinline__ void att_issue_rows(const StepParams& P, int l) {
  const mie_step_desc& d = ps_s.d;
  const StepGeom& g = ps_s.g;
  const mie_layer_desc& ly = layer_at(l);
  const int lane = threadIdx.x & 31;
  const int hd = d.head_dim, half = hd / 2, D = d.hidden_dim;
  const AttSplit a = att_split(g, hd, cx_s.pos);
  const uint32_t rb = (uint32_t)(D * sizeof(W));
  if (lane == 0) {
    fence_proxy_async_smem();  // earlier generic reads of these buffers before the async writes
    const uint32_t nrows = a.att ? (uint32_t)(g.q_stage + 2 * a.nkp + a.nvd) : 0u;
    bar_arm(kBarAtt, nrows * rb + (ly.attn_norm_b ? 2 : 1) * rb);
  }
  __syncwarp();
  // one copy per lane: norm weights, q rows, k (both RoPE halves), v; lane 5
  // prefetches the q rows that are not staged into L2
  if (lane == 5 && a.att && g.q_stage < hd) {
    const uint8_t* q0 = static_cast<const uint8_t*>(ly.qkv_w) + ((size_t)a.h * hd + g.q_stage) * rb;
#pragma unroll 1
    for (uint32_t o = 0, nb = (uint32_t)(hd - g.q_stage) * rb; o < nb; o += kBulkMax)
      bulk_prefetch_l2(q0 + o, min(kBulkMax, nb - o));
  }
  if (lane > 4 || (lane > 0 && !a.att)) return;
  fence_proxy_async_smem();
  const uint8_t* w = static_cast<const uint8_t*>(ly.qkv_w);
  uint8_t* ks = smem_at<uint8_t>(g.sm_kvw);
  const size_t kbase = (size_t)(D + a.h * hd + a.p0) * rb, vbase = (size_t)(2 * D + a.h * hd + a.v0) * rb;
  if (lane == 0)
    norm_copy(smem_at<uint8_t>(g.sm_anw), ly.attn_norm_w, ly.attn_norm_b, rb, kBarAtt);
  else if (lane == 1)
    bulk_copy(smem_at<uint8_t>(g.sm_qw), w + (size_t)a.h * hd * rb, g.q_stage * rb, kBarAtt);
  else if (lane == 2)
    bulk_copy(ks, w + kbase, a.nkp * rb, kBarAtt);
  else if (lane == 3)
    bulk_copy(ks + (size_t)a.nkp * rb, w + kbase + (size_t)half * rb, a.nkp * rb, kBarAtt);
  else
    bulk_copy(ks + (size_t)2 * a.nkp * rb, w + vbase, a.nvd * rb, kBarAtt);
}

// Stage the first K/V chunk of this CTA's old tokens of layer l (whole warp).
template <typename KV>
__device__ __noinline__ void att_issue_kv(const StepParams& P, int l) {
  const StepGeom& g = ps_s.g;
  const AttSplit a = att_split(g, ps_s.d.head_dim, cx_s.pos);
  const int n0 = min(g.chunk_tok, a.t1 - a.t0);
  if (n0 <= 0) return;
  if ((threadIdx.x & 31) == 0) fence_proxy_async_smem();
  __syncwarp();
  kv_issue<KV>(ps_s.d, g, layer_at(l), a.h, a.t0, n0, kBarKv);
}

// Stage layer l's out_proj rows of this CTA, the router and the MoE norm
// weights -- or, for l == num_layers, the final norm weights, into the
// attention norm slot (one thread).
template <typename W>
__device__ __noinline__ void side_issue(const StepParams& P, int l) {
  const mie_step_desc& d = ps_s.d;
  const StepGeom& g = ps_s.g;
  const int D = d.hidden_dim, E = d.num_experts;
  const uint32_t rb = (uint32_t)(D * sizeof(W));
  uint8_t* dst = smem_at<uint8_t>(g.sm_moe);
  fence_proxy_async_smem();
  if (l == d.num_layers) {
    bar_arm(kBarSide, (d.final_norm_b ? 2 : 1) * rb);
    norm_copy(smem_at<uint8_t>(g.sm_anw), d.final_norm_w, d.final_norm_b, rb, kBarSide);
    return;
  }
  const mie_layer_desc& ly = layer_at(l);
  int r0, r1;
  split32(D, blockIdx.x, gridDim.x, &r0, &r1);
  bar_arm(kBarSide, (uint32_t)(r1 - r0 + E + (ly.moe_norm_b ? 2 : 1)) * rb);
  bulk_copy(dst, static_cast<const uint8_t*>(ly.out_w) + (size_t)r0 * rb, (r1 - r0) * rb, kBarSide);
  bulk_copy(dst + (size_t)g.nr_max * rb, ly.router_w, E * rb, kBarSide);
  norm_copy(dst + (size_t)(g.nr_max + E) * rb, ly.moe_norm_w, ly.moe_norm_b, rb, kBarSide);
}

// Stages [first, first + count) of this CTA's LM-head rows (one thread) into
// the ring, which spans the attention staging area and the expert area.
template <typename W>
__device__ __noinline__ void head_issue(const StepParams& P, int first, int count) {
  const mie_step_desc& d = ps_s.d;
  const StepGeom& g = ps_s.g;
  int v0h, v1h;
  split32(d.vocab, blockIdx.x, gridDim.x, &v0h, &v1h);
  const uint32_t rb = (uint32_t)(d.hidden_dim * sizeof(W));
  const int nst = (v1h - v0h + g.head_rows - 1) / g.head_rows;
  fence_proxy_async_smem();
#pragma unroll 1
  for (int i = first; i < first + count && i < nst; ++i) {
    const int slot = i % g.head_stages;
    const int r0 = v0h + i * g.head_rows, nrw = min(g.head_rows, v1h - r0);
    bar_arm(kBarHead + slot, nrw * rb);
    bulk_copy(smem_at<uint8_t>(g.sm_qw) + (size_t)slot * g.head_rows * rb,
              static_cast<const uint8_t*>(d.embedding) + (size_t)r0 * rb, nrw * rb, kBarHead + slot, true);
  }
}

// ---------------------------------------------------------------------------
// Compute routines (shared by all phases)
// ---------------------------------------------------------------------------
// out = norm(in) with weight w (and bias b, LayerNorm) staged in shared memory
// as W; in, out fp32 vectors in shared memory (may alias).  Ends with a barrier.
template <typename W>
__device__ __noinline__ void norm_smem(float* out, const float* in, int D, int norm, float eps, const W* w,
                                       const W* b) {
  __syncthreads();
  float s1 = 0.f, s2 = 0.f;
#pragma unroll 1
  for (int i = threadIdx.x; i < D; i += kST) {
    const float v = in[i];
    s1 += v;
    s2 = fmaf(v, v, s2);
  }
  if (norm == MIE_NORM_RMS) {
    const float rs = rsqrtf(block_sum(s2, red_s) / (float)D + eps);
#pragma unroll 1
    for (int i = threadIdx.x; i < D; i += kST) out[i] = (in[i] * rs) * Elem<W>::to_f(w[i]);
  } else if (norm == MIE_NORM_LAYER) {
    const float mean = block_sum(s1, red_s) / (float)D;
    float v = 0.f;
#pragma unroll 1
    for (int i = threadIdx.x; i < D; i += kST) {
      const float t = in[i] - mean;
      v = fmaf(t, t, v);
    }
    const float rs = rsqrtf(block_sum(v, red_s) / (float)D + eps);
#pragma unroll 1
    for (int i = threadIdx.x; i < D; i += kST) {
      float y = (in[i] - mean) * rs * Elem<W>::to_f(w[i]);
      if (b) y += Elem<W>::to_f(b[i]);
      out[i] = y;
    }
  } else if (out != in) {
#pragma unroll 1
    for (int i = threadIdx.x; i < D; i += kST) out[i] = in[i];
  }
  __syncthreads();
}

// dst = the D words of exchange buffer buf (tag `tag`), out = norm(dst) with
// weight w (bias b) in shared memory; with bar >= 0 the bulk copies of
// barrier bar (the weights) are waited for as well.  RMSNorm folds the sum of
// squares into the receive: one barrier covers the receive, the copy wait and
// the cross-warp partials, a second one the output.  Same arithmetic, in the
// same order, as recv + bar_wait + norm_smem (the path other norms take).
template <typename W>
__device__ __noinline__ bool recv_norm(const uint64_t* buf, int D, uint32_t tag, float* dst, float* out, int bar,
                                       int norm, float eps, const W* w, const W* b, uint64_t* hdr,
                                       int32_t* status) {
  if (norm != MIE_NORM_RMS) {
    if (!recv(buf, D, tag, dst, nullptr, hdr, status)) return false;
    if (bar >= 0 && !bar_wait(bar, hdr, status)) return false;
    norm_smem<W>(out, dst, D, norm, eps, w, b);
    return true;
  }
  float s2;
  int bad = recv_poll(buf, D, tag, dst, nullptr, hdr, status, &s2);
  s2 = warp_sum(s2);
  if ((threadIdx.x & 31) == 0) red_s[threadIdx.x >> 5] = s2;  // last read of red_s: behind a barrier
  bool waited = false;
  if (bar >= 0 && !bad) {
    waited = mbar_wait(&bars_s[bar], bar_done_s[bar] & 1u, status, wait_ns_s);
    if (!waited) {
      atomicExch(reinterpret_cast<unsigned long long*>(hdr + kHdrAbort), 1ull);
      bad = 1;
    }
  }
  if (__syncthreads_or(bad)) return false;
  if (waited && threadIdx.x == 0) bar_done_s[bar] += 1;
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < kSW; ++i) t += red_s[i];
  const float rs = rsqrtf(t / (float)D + eps);
#pragma unroll 1
  for (int i = threadIdx.x; i < D; i += kST) out[i] = (dst[i] * rs) * Elem<W>::to_f(w[i]);
  __syncthreads();
  return true;
}

// Rows w, w + kSW, ... of warp w, R rows per iteration (one partial sum per
// 16-byte vector and row; the R shuffle reductions interleave).
template <typename W, bool kGlobal, int R>
__device__ __forceinline__ void gemv_rows(const uint4* rows, int n, int nvec, const float* xr, float* out) {
  constexpr int PV = Elem<W>::kPerVec, NV = Seg<W>::kNV;
  const int lane = threadIdx.x & 31;
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll 1
  for (int r = threadIdx.x >> 5; r < n; r += R * kSW) {
    uint4 w[R][NV];
#pragma unroll
    for (int k = 0; k < R; ++k) {
      const int rk = r + k * kSW < n ? r + k * kSW : r;
      const uint4* rp = rows + (size_t)rk * nvec;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int v = lane + kWarp * j;
        if constexpr (kGlobal)
          w[k][j] = v < nvec ? __ldg(rp + v) : z;
        else
          w[k][j] = v < nvec ? rp[v] : z;
      }
    }
    float sum[R];
#pragma unroll
    for (int k = 0; k < R; ++k) {
      sum[k] = 0.f;
#pragma unroll
      for (int j = 0; j < NV; ++j) sum[k] += dot_vec(w[k][j], xr + j * PV, 0.f, (const W*)nullptr);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
      for (int k = 0; k < R; ++k) sum[k] += __shfl_xor_sync(0xffffffffu, sum[k], o);
    }
    if (lane == 0) {
#pragma unroll
      for (int k = 0; k < R; ++k)
        if (r + k * kSW < n) out[r + k * kSW] = sum[k];
    }
  }
}

// Rows longer than one register segment (nvec > Seg<W>::kVecs: the expert
// down rows of a large expert hidden size, read from global memory; staged
// rows are never that long): out[r] = row r . x for r < n, rows [0, split)
// from rows0 dotted with x0, rows [split, n) from rows1 with x1 (both slots'
// rows in one pass).  One row per warp per iteration, segment by segment, the
// next segment's weights loaded before the current one is multiplied; one
// partial sum per 16-byte vector as in gemv_rows.
template <typename W, bool kGlobal>
__device__ __noinline__ void gemv_seg(const uint4* rows0, const uint4* rows1, int split, int n, int nvec,
                                      const float* x0, const float* x1, float* out) {
  constexpr int PV = Elem<W>::kPerVec, NV = Seg<W>::kNV, SV = Seg<W>::kVecs;
  const int lane = threadIdx.x & 31;
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  const auto load = [&](const uint4* rp, int s0, uint4* w) {
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int v = s0 + lane + kWarp * j;
      if constexpr (kGlobal)
        w[j] = v < nvec ? __ldg(rp + v) : z;
      else
        w[j] = v < nvec ? rp[v] : z;
    }
  };
#pragma unroll 1
  for (int r = threadIdx.x >> 5; r < n; r += kSW) {
    const float* xb = r < split ? x0 : x1;
    const uint4* rp = r < split ? rows0 + (size_t)r * nvec : rows1 + (size_t)(r - split) * nvec;
    uint4 w[NV], wn[NV];
    load(rp, 0, w);
    float sum = 0.f;
#pragma unroll 1
    for (int s0 = 0; s0 < nvec; s0 += SV) {
      if (s0 + SV < nvec) load(rp, s0 + SV, wn);
      float xr[NV * PV];
      load_x_regs<W>(xr, xb + (size_t)s0 * PV, nvec - s0);
#pragma unroll
      for (int j = 0; j < NV; ++j) sum += dot_vec(w[j], xr + j * PV, 0.f, (const W*)nullptr);
#pragma unroll
      for (int j = 0; j < NV; ++j) w[j] = wn[j];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) out[r] = sum;
  }
}

// ---- fp32 rows: CUDA-core GEMV ----
// out[r] = rows[r] . x for r < n: rows of nvec 16-byte vectors (row stride
// nvec) in shared memory (kGlobal false) or global memory, x an fp32 vector
// in shared memory (rows [split, n) dot x1 when x1 is set, n <= kSW).  Warp w
// forms rows w, w + kSW, ...: two rows per iteration and one partial sum per
// 16-byte vector, so the FMA chains and the two shuffle reductions are
// independent of each other.  No barrier.
template <typename W, bool kGlobal>
__device__ __noinline__ void gemv(const uint4* rows, int n, int nvec, const float* x, float* out,
                                  const float* x1 = nullptr, int split = 0) {
  constexpr int PV = Elem<W>::kPerVec;
  if ((threadIdx.x >> 5) >= n) return;  // no rows for this warp
  // rows [split, n) dot x1 instead of x (n <= kSW: one row per warp)
  const float* xb = (x1 && (int)(threadIdx.x >> 5) >= split) ? x1 : x;
  float xr[Seg<W>::kNV * PV];
  load_x_regs<W>(xr, xb, nvec);
  if (Seg<W>::kNV <= 3 && n == 4 * kSW)
    gemv_rows<W, kGlobal, Seg<W>::kNV <= 3 ? 4 : 2>(rows, n, nvec, xr, out);  // LM-head stages: 4 rows per warp
#ifdef MIE_STEP_WIDE_TU
  else if (Seg<W>::kNV <= 3 && n == 3 * kSW)
    gemv_rows<W, kGlobal, Seg<W>::kNV <= 3 ? 3 : 2>(rows, n, nvec, xr, out);  // wide LM-head stages of 48 rows
#endif
  else
    gemv_rows<W, kGlobal, 2>(rows, n, nvec, xr, out);
}

template <typename W>
__device__ __forceinline__ void gemv_smem(const uint4* rows, int n, int nvec, const float* x, float* out,
                                          const float* x1 = nullptr, int split = 0) {
  gemv<W, false>(rows, n, nvec, x, out, x1, split);
}
template <typename W>
__device__ __forceinline__ void gemv_global(const uint4* rows, int n, int nvec, const float* x, float* out) {
  gemv<W, true>(rows, n, nvec, x, out);
}

// Online softmax of q over K/V chunks of this split's old tokens [t0, t1)
// (the first chunk was staged with the layer's attention inputs).  Leaves
// the split's running max / normaliser in cx_s.m / cx_s.l and the PV group
// partials in ab[0, kST).
template <typename KV, bool kWide>
__device__ __noinline__ bool att_core(const StepParams& P, int l, int h, int t0, int t1, const float* q, float* sc,
                                      float* ab) {
  const mie_step_desc& d = ps_s.d;
  const StepGeom& g = ps_s.g;
  const int tid = threadIdx.x, hd = d.head_dim, chunk = g.chunk_tok;
  constexpr int VPT = 16 / (int)sizeof(KV);
  // PV: Gp groups of hd threads (threads past Gp * hd idle)
  const int VPH = hd / VPT, Gp = kST / hd, gi = tid / hd, dcol = tid - gi * hd;
  // kWide: any piece count (else a power of two)
  const KV* ks = smem_at<const KV>(g.sm_kv);
  const KV* vs = ks + (size_t)chunk * hd;
  const float scale = d.attn_scale;
  float m_run = -INFINITY, l_run = 0.f, acc = 0.f;
  const int nchunks = (t1 - t0 + chunk - 1) / chunk;
#pragma unroll 1
  for (int ci = 0; ci < nchunks; ++ci) {
    const int ta = t0 + ci * chunk, n = min(chunk, t1 - ta);
    if (ci > 0) {
      __syncthreads();  // previous chunk no longer read
      if (tid < 32) {
        if (tid == 0) fence_proxy_async_smem();
        __syncwarp();
        kv_issue<KV>(d, g, layer_at(l), h, ta, n, kBarKv);
      }
    }
    STEP_STAMP(l, 19);
    // every thread waits for the chunk's copies itself; whether all waits
    // succeeded is agreed at the barrier of the max below
    const bool kv_ok = mbar_wait(&bars_s[kBarKv], bar_done_s[kBarKv] & 1u, d.status, wait_ns_s);
    if (!kv_ok) atomicExch(reinterpret_cast<unsigned long long*>(g.ll + kHdrAbort), 1ull);
    STEP_STAMP(l, 20);
    float mloc = -INFINITY;
#pragma unroll 1
    for (int t = kv_ok ? tid : n; t < n; t += kST) {
      const uint4* kr = reinterpret_cast<const uint4*>(ks + (size_t)t * hd);
      // four independent partial dots; the start piece rotates with t, which
      // spreads the threads of a warp over the banks
      float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
      // piece (jj + t) mod VPH: a mask for a power of two, else a wrap of
      // jj + (t mod VPH) < 2 VPH
      const int rot = kWide ? t % VPH : t;
      const auto wrap = [VPH](int j) { return kWide ? (j >= VPH ? j - VPH : j) : (j & (VPH - 1)); };
      int jj = 0;
#pragma unroll 1
      for (; jj + 4 <= VPH; jj += 4) {
        const int j0 = wrap(jj + rot), j1 = wrap(jj + 1 + rot);
        const int j2 = wrap(jj + 2 + rot), j3 = wrap(jj + 3 + rot);
        d0 = dot_vec(kr[j0], q + j0 * VPT, d0, (const KV*)nullptr);
        d1 = dot_vec(kr[j1], q + j1 * VPT, d1, (const KV*)nullptr);
        d2 = dot_vec(kr[j2], q + j2 * VPT, d2, (const KV*)nullptr);
        d3 = dot_vec(kr[j3], q + j3 * VPT, d3, (const KV*)nullptr);
      }
#pragma unroll 1
      for (; jj < VPH; ++jj) {
        const int j = wrap(jj + rot);
        d0 = dot_vec(kr[j], q + j * VPT, d0, (const KV*)nullptr);
      }
      const float v = ((d0 + d1) + (d2 + d3)) * scale;
      sc[t] = v;
      mloc = fmaxf(mloc, v);
    }
    STEP_STAMP(l, 21);
    // block max (red_s) and block sum (red2_s) in the order of block_max /
    // block_sum; each buffer is rewritten only after later barriers
    mloc = warp_max(mloc);
    if ((tid & 31) == 0) red_s[tid >> 5] = mloc;
    if (__syncthreads_or(!kv_ok)) return false;
    if (tid == 0) bar_done_s[kBarKv] += 1;
    float bmax = -INFINITY;
#pragma unroll
    for (int i = 0; i < kSW; ++i) bmax = fmaxf(bmax, red_s[i]);
    const float mn = fmaxf(m_run, bmax);
    STEP_STAMP(l, 22);
    const float alpha = m_run == -INFINITY ? 0.f : expf(m_run - mn);
    float ls = 0.f;
#pragma unroll 1
    for (int t = tid; t < n; t += kST) {
      const float pr = expf(sc[t] - mn);
      sc[t] = pr;
      ls += pr;
    }
    ls = warp_sum(ls);
    if ((tid & 31) == 0) red2_s[tid >> 5] = ls;
    __syncthreads();  // also orders the sc writes before the PV reads
    float bsum = 0.f;
#pragma unroll
    for (int i = 0; i < kSW; ++i) bsum += red2_s[i];
    l_run = l_run * alpha + bsum;
    m_run = mn;
    STEP_STAMP(l, 23);
    if (gi < Gp) {
      // four independent accumulation chains over this group's tokens
      float a1 = 0.f, a2 = 0.f, a3 = 0.f, a0 = 0.f;
      int t = gi;
#pragma unroll 1
      for (; t + 3 * Gp < n; t += 4 * Gp) {
        a0 = fmaf(sc[t], Elem<KV>::to_f(vs[(size_t)t * hd + dcol]), a0);
        a1 = fmaf(sc[t + Gp], Elem<KV>::to_f(vs[(size_t)(t + Gp) * hd + dcol]), a1);
        a2 = fmaf(sc[t + 2 * Gp], Elem<KV>::to_f(vs[(size_t)(t + 2 * Gp) * hd + dcol]), a2);
        a3 = fmaf(sc[t + 3 * Gp], Elem<KV>::to_f(vs[(size_t)(t + 3 * Gp) * hd + dcol]), a3);
      }
#pragma unroll 1
      for (; t < n; t += Gp) a0 = fmaf(sc[t], Elem<KV>::to_f(vs[(size_t)t * hd + dcol]), a0);
      acc = fmaf(acc, alpha, (a0 + a1) + (a2 + a3));
    }
    STEP_STAMP(l, 24);
  }
  __syncthreads();
  STEP_STAMP(l, 25);
  ab[tid] = gi < Gp ? acc : 0.f;
  if (tid == 0) {
    cx_s.m = m_run;
    cx_s.l = l_run;
  }
  return true;
}

// ---------------------------------------------------------------------------
// ATT + MERGE of layer l (see the file comment).
// ---------------------------------------------------------------------------
template <typename W, typename KV, bool kWide>
__device__ __noinline__ bool att_phase(const StepParams& P, int l) {
  const mie_step_desc& d = ps_s.d;
  const StepGeom& g = ps_s.g;
  const mie_layer_desc& ly = layer_at(l);
  constexpr int PV = Elem<W>::kPerVec;
  const int tid = threadIdx.x;
  const int D = d.hidden_dim, hd = d.head_dim, half = hd / 2, nvD = D / PV;
  uint64_t* ll = g.ll;
  const uint32_t tag = tag_of(l);
  const int par = l & 1;
  float* xs = smem_at<float>(g.sm_x);
  float* xn = smem_at<float>(g.sm_xn);
  const int pos = cx_s.pos;
  const AttSplit a = att_split(g, hd, pos);
  const int S = g.S, nkv = 2 * a.nkp + a.nvd;
  STEP_STAMP(l, 0);

  // wide: this thread's q / k / v bias, loaded while x arrives (added after
  // the GEMVs)
  float qkv_bias = 0.f;
  if constexpr (kWide) {
    if (ly.qkv_b && a.att) {
      if (tid < hd) qkv_bias = ldw<W>(ly.qkv_b, (int64_t)a.h * hd + tid);
      if (tid >= 128 && tid < 128 + nkv) {
        const int k = tid - 128;
        const int64_t row = k < a.nkp       ? (int64_t)D + a.h * hd + a.p0 + k
                            : k < 2 * a.nkp ? (int64_t)D + a.h * hd + half + a.p0 + (k - a.nkp)
                                            : 2 * (int64_t)D + a.h * hd + a.v0 + (k - 2 * a.nkp);
        qkv_bias = ldw<W>(ly.qkv_b, row);
      }
    }
  }
  // ---- x: token embedding (layer 0) or exchange A; norm ----
  const W* nw = smem_at<const W>(g.sm_anw);
  if (l == 0) {
    const int64_t tok = cx_s.tok;
#pragma unroll 1
    for (int i = tid; i < D; i += kST) {
      float v = ldw<W>(d.embedding, tok * D + i);
      if (d.pos_embedding) v += ldw<W>(d.pos_embedding, (int64_t)pos * D + i);
      xs[i] = v;
    }
    if (!bar_wait(kBarAtt, ll, d.status)) return false;
    norm_smem<W>(xn, xs, D, d.norm, d.eps, nw, ly.attn_norm_b ? nw + D : nullptr);
  } else if (!recv_norm<W>(ll + g.off_a[par], D, tag, xs, xn, kBarAtt, d.norm, d.eps, nw,
                           ly.attn_norm_b ? nw + D : nullptr, ll, d.status)) {
    return false;
  }
  STEP_STAMP(l, 2);
  if (!a.att) return true;

  // ---- q rows of head h and this CTA's k / v rows: qk[0, hd) = q, qk[hd, hd + nkv) = k, v ----
  float* qk = smem_at<float>(g.sm_qk);
  if (g.q_stage == hd && g.sm_kvw == g.sm_qw + (uint32_t)(hd * nvD * 16)) {
    gemv_smem<W>(smem_at<const uint4>(g.sm_qw), hd + nkv, nvD, xn, qk);  // q and k / v rows are adjacent
  } else {
    gemv_smem<W>(smem_at<const uint4>(g.sm_qw), g.q_stage, nvD, xn, qk);
    // the q rows that did not fit in shared memory (prefetched into L2 with
    // the staging); bf16 weights in the narrow geometry stage every q row
    if constexpr (sizeof(W) == 4 || kWide)
      if (g.q_stage < hd)
        gemv_global<W>(rowp(ly.qkv_w, (int64_t)a.h * hd + g.q_stage, (int64_t)nvD * 16), hd - g.q_stage, nvD, xn,
                       qk + g.q_stage);
    gemv_smem<W>(smem_at<const uint4>(g.sm_kvw), nkv, nvD, xn, qk + hd);
  }
  __syncthreads();
  STEP_STAMP(l, 3);
  // bias; RoPE of q (pairs j, j + hd/2) and of this CTA's k pairs; k / v
  // rounded to the cache type and stored into the slot of the new token
  float* kv = qk + hd;
  if (kWide && ly.qkv_b) {
    if (tid < hd) qk[tid] += qkv_bias;
    if (tid >= 128 && tid < 128 + nkv) kv[tid - 128] += qkv_bias;
    __syncthreads();
  } else if (ly.qkv_b) {
    if (tid < hd) qk[tid] += ldw<W>(ly.qkv_b, (int64_t)a.h * hd + tid);
    if (tid >= 128 && tid < 128 + nkv) {
      const int k = tid - 128;
      const int64_t row = k < a.nkp       ? (int64_t)D + a.h * hd + a.p0 + k
                          : k < 2 * a.nkp ? (int64_t)D + a.h * hd + half + a.p0 + (k - a.nkp)
                                          : 2 * (int64_t)D + a.h * hd + a.v0 + (k - 2 * a.nkp);
      kv[k] += ldw<W>(ly.qkv_b, row);
    }
    __syncthreads();
  }
  const float* cs = d.rope_cos ? d.rope_cos + (int64_t)pos * half : nullptr;
  const float* sn = d.rope_sin ? d.rope_sin + (int64_t)pos * half : nullptr;
  if (cs && tid < half) {
    const float x1 = qk[tid], x2 = qk[tid + half], cv = cs[tid], sv = sn[tid];
    qk[tid] = x1 * cv - x2 * sv;
    qk[tid + half] = x2 * cv + x1 * sv;
  }
  const int64_t slot = cx_s.slot + (int64_t)a.h * d.kv_stride_head;
  if (tid >= 128 && tid < 128 + a.nkp) {
    const int k = tid - 128, i = a.p0 + k;
    float x1 = kv[k], x2 = kv[a.nkp + k];
    if (cs) {
      const float y1 = x1 * cs[i] - x2 * sn[i];
      const float y2 = x2 * cs[i] + x1 * sn[i];
      x1 = y1;
      x2 = y2;
    }
    const KV k1 = Elem<KV>::from_f(x1), k2 = Elem<KV>::from_f(x2);
    KV* kc = static_cast<KV*>(ly.k_cache);
    kc[slot + i] = k1;
    kc[slot + i + half] = k2;
    kv[k] = Elem<KV>::to_f(k1);
    kv[a.nkp + k] = Elem<KV>::to_f(k2);
  } else if (tid >= 256 && tid < 256 + a.nvd) {
    const int k = tid - 256;
    const KV vv = Elem<KV>::from_f(kv[2 * a.nkp + k]);
    static_cast<KV*>(ly.v_cache)[slot + a.v0 + k] = vv;
    kv[2 * a.nkp + k] = Elem<KV>::to_f(vv);
  }
  __syncthreads();
  STEP_STAMP(l, 4);

  // ---- attention over the old tokens ----
  float* ab = smem_at<float>(g.sm_acc);
  if (!att_core<KV, kWide>(P, l, a.h, a.t0, a.t1, qk, smem_at<float>(g.sm_sc), ab)) return false;
  __syncthreads();  // staged rows, K/V and ab complete
  STEP_STAMP(l, 5);
  uint64_t* be = ll + g.off_b[par] + (int64_t)(a.h * S + a.s) * (3 + hd);
  const int Gp = kST / hd;
  if (tid < hd) {
    float s = 0.f;
#pragma unroll 1
    for (int k = 0; k < Gp; ++k) s += ab[k * hd + tid];
    ll_put(be + 3 + tid, s, tag);
  } else if (tid == hd) {
    // this CTA's share of q . k_new (k rounded to the cache type)
    float sp = 0.f;
#pragma unroll 1
    for (int k = 0; k < a.nkp; ++k) {
      sp = fmaf(qk[a.p0 + k], kv[k], sp);
      sp = fmaf(qk[a.p0 + k + half], kv[a.nkp + k], sp);
    }
    ll_put(be + 0, cx_s.m, tag);
    ll_put(be + 1, cx_s.l, tag);
    ll_put(be + 2, sp, tag);
  }
  STEP_STAMP(l, 6);

  // ---- MERGE: ab[0, 3S) = (m, l, sp) of every split, ab[3S, 3S + S nvd) = acc of my dims ----
  if (a.nvd == 0) return true;
  const int nm = 3 * S, nvd = a.nvd, nwords = nm + S * nvd;
#pragma unroll 1
  for (int i = tid; i < nwords; i += kST) {
    int at;
    if (i < nm) {
      at = (i / 3) * (3 + hd) + (i % 3);
    } else {
      const int j = i - nm, sp = j / nvd;
      at = sp * (3 + hd) + 3 + a.v0 + (j - sp * nvd);
    }
    gat_s[i] = at;
  }
  __syncthreads();  // gather indices ready, ab (PV groups) fully read
  if (!recv(ll + g.off_b[par] + (int64_t)a.h * S * (3 + hd), nwords, tag, ab, gat_s, ll, d.status)) return false;
  STEP_STAMP(l, 7);
  if (tid < 32) {
    // warp 0: split weights w_k = e^(m_k - M) with the new token as one more
    // term (score q.k_new, value v_new), M the largest score; lane k forms
    // w_k of splits k, k + 32, ... (S broadcast reads for M), then lane d < nvd
    // the output of dim v0 + d, summing the splits in order
    float sp = 0.f, mx = -INFINITY;
#pragma unroll 4
    for (int k = 0; k < S; ++k) {
      sp += ab[3 * k + 2];
      mx = fmaxf(mx, ab[3 * k]);
    }
    const float snew = sp * d.attn_scale;
    const float M = fmaxf(mx, snew);
    float* wk = smem_at<float>(g.sm_sc);  // scores scratch, free after the attention core
#pragma unroll 1
    for (int k = tid; k < S; k += 32) {
      const float mk = ab[3 * k];
      wk[k] = mk == -INFINITY ? 0.f : expf(mk - M);
    }
    __syncwarp();
    if (tid < nvd) {
      const float wn = expf(snew - M);
      float den = 0.f, num = 0.f;
#pragma unroll 4
      for (int k = 0; k < S; ++k) {
        const float w = wk[k];
        den = fmaf(ab[3 * k + 1], w, den);
        num = fmaf(ab[nm + k * nvd + tid], w, num);
      }
      num = fmaf(wn, kv[2 * a.nkp + tid], num);
      ll_put(ll + g.off_c[par] + (int64_t)a.h * hd + a.v0 + tid, num / (den + wn), tag);
    }
  }
  // the PROJ threads start polling o only after this CTA's merge: polls
  // issued early only load the lines the producers are about to write
  if (tid < kProjThreads) bar_sync_part();
  STEP_STAMP(l, 15);
  return true;
}

// ---------------------------------------------------------------------------
// PROJ: x_mid rows = x + out_proj(o) (+ bias) -> exchange D.
// ---------------------------------------------------------------------------
template <typename W, typename KV, bool kWide>
__device__ __noinline__ bool proj_phase(const StepParams& P, int l) {
  const mie_step_desc& d = ps_s.d;
  const StepGeom& g = ps_s.g;
  const mie_layer_desc& ly = layer_at(l);
  constexpr int PV = Elem<W>::kPerVec;
  const int tid = threadIdx.x, D = d.hidden_dim, nvD = D / PV;
  uint64_t* ll = g.ll;
  const uint32_t tag = tag_of(l);
  int r0, r1;
  split32(D, blockIdx.x, gridDim.x, &r0, &r1);
  const int nr = r1 - r0;
  float* ob = smem_at<float>(g.sm_o);
  float* ab = smem_at<float>(g.sm_acc);
  // While o is on its way: stage the next layer's attention inputs (the
  // attention staging area is free since this layer's attention), or the
  // first LM-head rows after the last layer.
  const int warp = tid >> 5;
  STEP_STAMP_T(l, 16, kST - 32);
  if (tid >= kProjThreads) {
    // the last two warps: copy issue only; they meet the others at the next
    // phase's first barrier
    if (warp == kSW - 1) {
      if (l + 1 < d.num_layers)
        att_issue_rows<W>(P, l + 1);
      else if ((tid & 31) == 0)
        head_issue<W>(P, 0, g.head_early);  // stages clear of the expert area
    } else {
      if (l + 1 < d.num_layers) att_issue_kv<KV>(P, l + 1);
      if (l + 2 < d.num_layers) layer_fetch(P, l + 2, kST - 64);  // into the slot of layer l - 2
    }
    STEP_STAMP_T(l, 17, kST - 32);
    return true;
  }
  STEP_STAMP(l, 18);
  // a failed wait raised the abort word: the next receive then fails for
  // every thread of every CTA, so no barrier is needed to agree here
  // wide: the bias of this thread's row, loaded while o arrives
  const float out_bias = kWide && ly.out_b && tid < nr ? ldw<W>(ly.out_b, r0 + tid) : 0.f;
  if (!recv_part(ll + g.off_c[l & 1], D, tag, ob, kBarSide, ll, d.status)) return true;
  STEP_STAMP(l, 8);
  gemv_smem<W>(smem_at<const uint4>(g.sm_moe), nr, nvD, ob, ab);  // nr <= 14 rows: warps < 14
  bar_sync_part();
  if (tid < nr) {
    const int r = r0 + tid;
    float y = ab[tid];
    if (kWide)
      y += out_bias;
    else if (ly.out_b)
      y += ldw<W>(ly.out_b, r);
    ll_put(ll + g.off_d[l & 1] + r, smem_at<float>(g.sm_x)[r] + y, tag);
  }
  STEP_STAMP(l, 9);
  return true;
}

// Warp 0 of a wide-geometry CTA, right after routing: the selected experts'
// rows of this CTA -- gate (and up) rows of its units [u0, u1), down rows of
// its output rows -- prefetched into L2 for the GEMVs that read them from
// global memory (lanes 0-3: up rows of each matrix and slot; lanes 8-9: down
// rows of each slot).
template <typename W>
__device__ __noinline__ void moe_prefetch(int l, int sel0, int sel1) {
  const mie_step_desc& d = ps_s.d;
  const mie_layer_desc& ly = layer_at(l);
  const int tid = threadIdx.x, D = d.hidden_dim, Hx = d.expert_hidden_dim;
  const int nmat = d.act == MIE_ACT_SWIGLU ? 2 : 1;
  const uint32_t rbD = (uint32_t)(D * sizeof(W)), rbH = (uint32_t)(Hx * sizeof(W));
  const uint8_t* src = nullptr;
  uint32_t nb = 0;
  if (tid < 2 * nmat) {
    int u0, u1;
    split32(2 * Hx, blockIdx.x, gridDim.x, &u0, &u1);
    const int m = tid >> 1, k = tid & 1;
    const int ua = max(u0, k * Hx), ub = min(u1, (k + 1) * Hx);
    if (ub > ua) {
      src = static_cast<const uint8_t*>(m ? ly.w3 : ly.w1) + ((size_t)(k ? sel1 : sel0) * Hx + ua - k * Hx) * rbD;
      nb = (uint32_t)(ub - ua) * rbD;
    }
  } else if (tid >= 8 && tid < 10) {
    int r0, r1;
    split32(D, blockIdx.x, gridDim.x, &r0, &r1);
    const int k = tid - 8;
    src = static_cast<const uint8_t*>(ly.w2) + ((size_t)(k ? sel1 : sel0) * D + r0) * rbH;
    nb = (uint32_t)(r1 - r0) * rbH;
  }
#pragma unroll 1
  for (uint32_t o = 0; o < nb; o += kBulkMax) bulk_prefetch_l2(src + o, min(kBulkMax, nb - o));
}

// ---------------------------------------------------------------------------
// UP + DOWN: x_mid -> norm -> router -> top-2 -> selected experts -> x of
// layer l + 1 (exchange A).  bf16 weights: the selected experts' rows of this
// CTA are bulk-copied into shared memory right after routing; fp32 weights:
// read from global memory by the GEMV.  kWide (shapes whose expert rows do not
// fit in shared memory): read from global memory after an L2 prefetch, down
// rows longer than one register segment multiplied segment by segment.
// ---------------------------------------------------------------------------
template <typename W, bool kWide>
__device__ __noinline__ bool moe_phase(const StepParams& P, int l) {
  const mie_step_desc& d = ps_s.d;
  const StepGeom& g = ps_s.g;
  const mie_layer_desc& ly = layer_at(l);
  constexpr int PV = Elem<W>::kPerVec;
  constexpr bool kStaged = sizeof(W) == 2 && !kWide;
  const int tid = threadIdx.x;
  const int D = d.hidden_dim, Hx = d.expert_hidden_dim, E = d.num_experts, nvD = D / PV, nvH = Hx / PV;
  const int64_t rbD = (int64_t)D * sizeof(W), rbH = (int64_t)Hx * sizeof(W);
  const bool swiglu = d.act == MIE_ACT_SWIGLU;
  const int nmat = swiglu ? 2 : 1;
  uint64_t* ll = g.ll;
  const uint32_t tag = tag_of(l);
  const int par = l & 1;
  float* xm = smem_at<float>(g.sm_xm);
  float* xn = smem_at<float>(g.sm_xn);
  float* hb = smem_at<float>(g.sm_h);
  float* ab = smem_at<float>(g.sm_acc);
  uint8_t* ms = smem_at<uint8_t>(g.sm_moe);
  int u0, u1, r0, r1;
  split32(2 * Hx, blockIdx.x, gridDim.x, &u0, &u1);  // up units
  split32(D, blockIdx.x, gridDim.x, &r0, &r1);       // output rows
  const int nu = u1 - u0, nr = r1 - r0;

  const W* nw = reinterpret_cast<const W*>(ms + (size_t)(g.nr_max + E) * rbD);
  if (!recv_norm<W>(ll + g.off_d[par], D, tag, xm, xn, -1, d.norm, d.eps, nw, ly.moe_norm_b ? nw + D : nullptr, ll,
                    d.status))
    return false;
  STEP_STAMP(l, 10);
  gemv_smem<W>(reinterpret_cast<const uint4*>(ms + (size_t)g.nr_max * rbD), E, nvD, xn, ab);
  __syncthreads();
  // top-2 over the router logits, by every thread (E broadcast reads, no
  // exchange): largest logit, ties to the lower id -- a repeated argmax
  // scanning ascending ids with a strict '>' -- and the softmax of the pair
  int sel0 = 0;
  float bv = ab[0];
#pragma unroll 1
  for (int e = 1; e < E; ++e)
    if (ab[e] > bv) {
      bv = ab[e];
      sel0 = e;
    }
  int sel1 = sel0 == 0 ? 1 : 0;
  float cv = ab[sel1];
#pragma unroll 1
  for (int e = sel1 + 1; e < E; ++e)
    if (e != sel0 && ab[e] > cv) {
      cv = ab[e];
      sel1 = e;
    }
  const float e1 = expf(cv - bv);
  const float wt0 = 1.0f / (1.0f + e1), wt1 = e1 / (1.0f + e1);
  if constexpr (kStaged) {
    // the selected experts' rows of this CTA -> shared memory (over the
    // out_proj / router / norm rows, all read by now): gate rows of units
    // [u0, u1), up rows (SwiGLU), down rows (slot 0 then slot 1); thread c of
    // warp 0 issues copy c after thread 0 armed the barriers
    if (tid == 0) {
      fence_proxy_async_smem();
      bar_arm(kBarMoe, (uint32_t)(nmat * nu * rbD));  // up rows
      bar_arm(kBarDown, (uint32_t)(2 * nr * rbH));    // down rows, needed after exchange E
    }
    if (tid < 32) {
      __syncwarp();
      if (tid < 2 * nmat) {
        const int m = tid >> 1, k = tid & 1;
        const uint8_t* w = static_cast<const uint8_t*>(m ? ly.w3 : ly.w1);
        const int ua = max(u0, k * Hx), ub = min(u1, (k + 1) * Hx);
        fence_proxy_async_smem();
        if (ub > ua)
          bulk_copy(ms + (size_t)(m * nu + ua - u0) * rbD, w + ((size_t)(k ? sel1 : sel0) * Hx + ua - k * Hx) * rbD,
                    (uint32_t)((ub - ua) * rbD), kBarMoe);
      } else if (tid >= 8 && tid < 10) {
        const int k = tid - 8;
        fence_proxy_async_smem();
        bulk_copy(ms + (size_t)nmat * nu * rbD + (size_t)k * nr * rbH,
                  static_cast<const uint8_t*>(ly.w2) + ((size_t)(k ? sel1 : sel0) * D + r0) * rbH,
                  (uint32_t)(nr * rbH), kBarDown);
      }
    }
  }
  if constexpr (kWide) {
    if (tid < 32) moe_prefetch<W>(l, sel0, sel1);
  }
  STEP_STAMP(l, 11);
  // up units: gate (and up) rows -> ab[0, nmat * nu)
  if constexpr (kStaged) {
    if (!bar_wait(kBarMoe, ll, d.status)) return false;
    gemv_smem<W>(reinterpret_cast<const uint4*>(ms), nmat * nu, nvD, xn, ab);
  } else {
#pragma unroll 1
    for (int m = 0; m < nmat; ++m) {
      const void* w = m ? ly.w3 : ly.w1;
#pragma unroll 1
      for (int k = 0; k < 2; ++k) {
        const int ua = max(u0, k * Hx), ub = min(u1, (k + 1) * Hx);
        if (ub > ua)
          gemv_global<W>(rowp(w, (int64_t)(k ? sel1 : sel0) * Hx + ua - k * Hx, rbD), ub - ua, nvD, xn,
                         ab + m * nu + (ua - u0));
      }
    }
  }
  __syncthreads();
  const bool side_now = kStaged && l + 1 < d.num_layers && g.nr_max + E + 2 <= nmat * nu;
  if (side_now && tid == kST - 1) side_issue<W>(P, l + 1);
  if (tid < nu) {
    const int u = u0 + tid, k = u / Hx;
    const int64_t row = (int64_t)(k ? sel1 : sel0) * Hx + (u - k * Hx);
    float gv = ab[tid];
    if (ly.b1) gv += ldw<W>(ly.b1, row);
    ll_put(ll + g.off_e[par] + u, swiglu ? silu(gv) * ab[nu + tid] : gelu_erf(gv), tag);
  }
  STEP_STAMP(l, 12);

  // ---- DOWN ----
  if (!recv(ll + g.off_e[par], 2 * Hx, tag, hb, nullptr, ll, d.status)) return false;
  STEP_STAMP(l, 13);
  // the next layer's out_proj / router / norm rows go over the consumed up
  // rows while the down GEMV runs (warps < 2 nr), issued by the last thread,
  // when they fit there; else after the down GEMV
  if constexpr (kStaged) {
    if (!bar_wait(kBarDown, ll, d.status)) return false;
  }
  if (kStaged && 2 * nr <= kSW) {
    // both slots' down rows (adjacent in shared memory) in one pass: rows
    // [0, nr) dot h of slot 0, rows [nr, 2 nr) dot h of slot 1
    gemv_smem<W>(reinterpret_cast<const uint4*>(ms + (size_t)nmat * nu * rbD), 2 * nr, nvH, hb, ab, hb + Hx, nr);
  } else if (kWide && nvH > Seg<W>::kVecs) {
    // rows longer than one register segment, both slots in one pass
    gemv_seg<W, true>(rowp(ly.w2, (int64_t)sel0 * D + r0, rbH), rowp(ly.w2, (int64_t)sel1 * D + r0, rbH), nr, 2 * nr,
                      nvH, hb, hb + Hx, ab);
  } else {
#pragma unroll 1
    for (int k = 0; k < 2; ++k) {
      if constexpr (kStaged)
        gemv_smem<W>(reinterpret_cast<const uint4*>(ms + (size_t)nmat * nu * rbD + (size_t)k * nr * rbH), nr, nvH,
                     hb + (size_t)k * Hx, ab + k * nr);
      else
        gemv_global<W>(rowp(ly.w2, (int64_t)(k ? sel1 : sel0) * D + r0, rbH), nr, nvH, hb + (size_t)k * Hx,
                       ab + k * nr);
    }
  }
  __syncthreads();
  if (tid < nr) {
    const int r = r0 + tid;
    float y = xm[r];
#pragma unroll 1
    for (int k = 0; k < 2; ++k) {
      float v = ab[k * nr + tid];
      if (ly.b2) v += ldw<W>(ly.b2, (int64_t)(k ? sel1 : sel0) * D + r);
      y = fmaf(k ? wt1 : wt0, v, y);
    }
    ll_put(ll + g.off_a[(l + 1) & 1] + r, y, tag_of(l + 1));
    if (l == d.num_layers - 1) d.x[r] = y;
  }
  // else stage the next layer's out_proj / router / norm rows (or the final
  // norm) now, from a thread without an output row
  if (tid == kST - 1 && !side_now) {
    side_issue<W>(P, l + 1);
    // after the last layer the expert area is free: the remaining first stages
    // of the LM-head ring
    if (l + 1 == d.num_layers) head_issue<W>(P, g.head_early, g.head_stages - g.head_early);
  }
  STEP_STAMP(l, 14);
  return true;
}

// ---------------------------------------------------------------------------
// HEAD: x_L -> final norm -> tied LM head -> argmax + device bookkeeping.
// The CTA's vocab rows stream through a ring of head_stages stages of
// head_rows rows over the attention and expert staging areas; the first
// stages were requested during the last layer.
// ---------------------------------------------------------------------------
// Last CTA of the LM head: publish the step's token (device state, token
// log, EOS flag) and reset the head's counter for the next step (one thread).
__device__ __noinline__ void head_finish(int bi) {
  const mie_step_desc& d = ps_s.d;
  if (bi < 0 || bi >= d.vocab) {  // every logit NaN
    set_status(d.status, MIE_ERR_RANGE);
    bi = 0;
  }
  *d.token = bi;
  *d.pos = cx_s.pos + 1;
  if (d.tokens_log && d.log_count) {
    const int k = cx_s.log_k;  // read at the start of the step; only this step writes it
    if (k < d.log_capacity) d.tokens_log[k] = bi;
    *d.log_count = k + 1;
  }
  if (d.done && bi == d.eos_id) *d.done = 1;
  *d.lm_counter = 0u;
  __threadfence();
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(ps_s.g.ll + kHdrStep), "l"((uint64_t)cx_s.step)
               : "memory");
}

// Sampling with top-k (model.py:604-613): this CTA's logits (headv_s) sorted,
// its top_k candidates published; the last CTA sorts all candidates, keeps
// the logits >= the top_k-th largest and draws among them by Gumbel-max.
__device__ __noinline__ bool head_sample_topk(int v0h, int v1h, uint64_t seed, float inv_t) {
  const mie_step_desc& d = ps_s.d;
  const StepGeom& g = ps_s.g;
  const int tid = threadIdx.x, c = blockIdx.x, G = gridDim.x, K = d.sample_top_k, n = v1h - v0h;
  uint64_t* keys = smem_at<uint64_t>(g.sm_qw);  // the LM-head ring: every stage consumed
  const float* headv = smem_at<const float>(g.sm_h);  // this CTA's logits (the h vector is free in the head)
  __syncthreads();
#pragma unroll 1
  for (int i = tid; i < kStepHeadRowsMax; i += kST) keys[i] = i < n ? logit_key(headv[i], v0h + i) : 0ull;
  sort_keys_desc(keys, kStepHeadRowsMax);
  uint64_t* cand = g.ll + g.off_cand + (int64_t)c * kStepTopKMax;
  if (tid < K) cand[tid] = keys[tid];
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    cx_s.last = atom_add_acq_rel_gpu(d.lm_counter, 1u) == (uint32_t)(G - 1);
  }
  __syncthreads();
  if (!cx_s.last) return true;
  __threadfence();
  const int m = G * K;
  int n2 = 1;
  while (n2 < m) n2 <<= 1;
#pragma unroll 1
  for (int i = tid; i < n2; i += kST)
    keys[i] = i < m ? __ldcg(g.ll + g.off_cand + (int64_t)(i / K) * kStepTopKMax + i % K) : 0ull;
  sort_keys_desc(keys, n2);
  const float theta = key_logit(keys[K - 1]);
  float best_v = -INFINITY;
  int best_i = 0x7fffffff;
#pragma unroll 1
  for (int i = tid; i < m; i += kST) {
    const uint64_t k = keys[i];
    const float v = key_logit(k);
    if (k == 0ull || !(v >= theta)) continue;
    const int row = key_row(k);
    const float sc = v * inv_t + gumbel(seed, cx_s.pos, row);
    if (better(sc, row, best_v, best_i)) {
      best_v = sc;
      best_i = row;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
    if (better(ov, oi, best_v, best_i)) {
      best_v = ov;
      best_i = oi;
    }
  }
  if ((tid & 31) == 0) {
    bestv_s[tid >> 5] = best_v;
    besti_s[tid >> 5] = best_i;
  }
  __syncthreads();
  if (tid == 0) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll 1
    for (int w = 0; w < kSW; ++w)
      if (better(bestv_s[w], besti_s[w], bv, bi)) {
        bv = bestv_s[w];
        bi = besti_s[w];
      }
    head_finish(bi);
  }
  return true;
}

template <typename W, bool kWide>
__device__ __noinline__ bool head_phase(const StepParams& P) {
  const mie_step_desc& d = ps_s.d;
  const StepGeom& g = ps_s.g;
  constexpr int PV = Elem<W>::kPerVec;
  const int G = gridDim.x, c = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int D = d.hidden_dim, nvD = D / PV, V = d.vocab, Lnum = d.num_layers;
  uint64_t* ll = g.ll;
  float* xs = smem_at<float>(g.sm_x);
  float* xn = smem_at<float>(g.sm_xn);
  float* ab = smem_at<float>(g.sm_acc);
  STEP_STAMP(Lnum, 0);
  int v0h, v1h;
  split32(V, c, G, &v0h, &v1h);
  const int nst = (v1h - v0h + g.head_rows - 1) / g.head_rows;
  const W* nw = smem_at<const W>(g.sm_anw);
  // wide: the LM-head bias of this CTA's vocab rows into the h vector's
  // shared memory (free in the head) while x arrives; the top-k sampler's
  // logits later overwrite each entry after its own bias was read
  float* hbias = smem_at<float>(g.sm_h);
  const bool bias_smem = kWide && d.lm_bias && g.head_bias_smem;
  if (bias_smem)
#pragma unroll 1
    for (int i = tid; i < v1h - v0h; i += kST) hbias[i] = ldw<W>(d.lm_bias, v0h + i);
  if (!recv_norm<W>(ll + g.off_a[Lnum & 1], D, tag_of(Lnum), xs, xn, kBarSide, d.norm, d.eps, nw,
                    d.final_norm_b ? nw + D : nullptr, ll, d.status))
    return false;
  STEP_STAMP(Lnum, 1);
  // greedy (temperature 0): argmax of the logits; sampling: argmax of
  // logit / T + Gumbel noise over every token, or the top-k sampler
  const bool sample = d.sample_temperature > 0.f, topk = sample && d.sample_top_k > 0;
  const uint64_t seed = sample ? __ldcg(reinterpret_cast<const unsigned long long*>(d.sample_seed)) : 0ull;
  const float inv_t = sample ? 1.0f / d.sample_temperature : 0.f;
  float best_v = -INFINITY;
  int best_i = 0x7fffffff;
#pragma unroll 1
  for (int i = 0; i < nst; ++i) {
    const int slot = i % g.head_stages;
    if (!bar_wait(kBarHead + slot, ll, d.status)) return false;
    const int r0 = v0h + i * g.head_rows, nrw = min(g.head_rows, v1h - r0);
    gemv_smem<W>(smem_at<const uint4>(g.sm_qw) + (size_t)slot * g.head_rows * nvD, nrw, nvD, xn, ab);
    __syncthreads();  // stage no longer read, ab complete
    if (tid == 0 && i + g.head_stages < nst) head_issue<W>(P, i + g.head_stages, 1);
    if (tid < nrw) {
      float v = ab[tid];
      const int row = r0 + tid;
      if (bias_smem)
        v += hbias[row - v0h];
      else if (d.lm_bias)
        v += ldw<W>(d.lm_bias, row);
      if (d.logits) d.logits[row] = v;
      if (topk) {
        smem_at<float>(g.sm_h)[row - v0h] = v;
      } else {
        const float sc = sample ? v * inv_t + gumbel(seed, cx_s.pos, row) : v;
        if (better(sc, row, best_v, best_i)) {
          best_v = sc;
          best_i = row;
        }
      }
    }
  }
  STEP_STAMP(Lnum, 2);
  if (topk) return head_sample_topk(v0h, v1h, seed, inv_t);
  // CTA argmax: (value, lower index) is a total order, so the reduction
  // order does not change the result
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
  __syncthreads();
  if (tid == 0) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll 1
    for (int w = 0; w < kSW; ++w)
      if (better(bestv_s[w], besti_s[w], bv, bi)) {
        bv = bestv_s[w];
        bi = besti_s[w];
      }
    d.lm_partial_val[c] = bv;
    d.lm_partial_idx[c] = bi;
    // the release half of the atomic orders this thread's two stores before it
    cx_s.last = atom_add_acq_rel_gpu(d.lm_counter, 1u) == (uint32_t)(G - 1);
  }
  __syncthreads();
  if (!cx_s.last || warp != 0) return true;
  __threadfence();
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  // eight partials per lane per round, loaded before any is compared
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
  STEP_STAMP(Lnum, 5);
  return true;
}

// Wait (bounded by limit_ns) until the start gate *gate is nonzero; false when
// it stayed closed.  Acquire: what the gate's writer wrote before opening it is
// visible afterwards.
__device__ __noinline__ bool gate_open(const int32_t* gate, unsigned long long limit_ns) {
  const unsigned long long t0 = global_ns();
#pragma unroll 1
  while (ld_acquire_gpu(reinterpret_cast<const uint32_t*>(gate)) == 0u)
    if (global_ns() - t0 > limit_ns) return false;
  return true;
}

template <typename W, typename KV, bool kWide>
__global__ void __launch_bounds__(kST, 1) step_kernel(const __grid_constant__ StepParams P) {
  STEP_STAMP(P.d.num_layers, 3);
  // Under programmatic dependent launch the next step's CTAs may take each SM
  // this grid's CTAs leave (one CTA fills an SM, so none starts earlier); they
  // stage their first weights, then wait for this grid to complete.
  pdl_trigger();
  {
    // parameters -> shared memory: descriptor and geometry, layers 0 .. 3
    constexpr int kWords = (int)(sizeof(StepShared) / 8);
    static_assert(sizeof(mie_step_desc) % 8 == 0 && sizeof(StepGeom) % 8 == 0, "8-byte words");
    const int i = threadIdx.x;
    if (i < kWords) {
      const uint64_t* src = i < (int)(sizeof(mie_step_desc) / 8)
                                ? reinterpret_cast<const uint64_t*>(&P.d) + i
                                : reinterpret_cast<const uint64_t*>(&P.g) + (i - (int)(sizeof(mie_step_desc) / 8));
      reinterpret_cast<uint64_t*>(&ps_s)[i] = *src;
    }
#pragma unroll 1
    for (int l = 0; l < kLayerSlots && l < P.d.num_layers; ++l) layer_fetch(P, l, 128 + 16 * l);
    if (threadIdx.x == 0) {
      cx_s.pos = 0;
#pragma unroll 1
      for (int b = 0; b < kNumBars; ++b) {
        mbar_init(&bars_s[b], 1);
        bar_armed_s[b] = bar_done_s[b] = 0;
      }
      fence_barrier_init();
    }
    __syncthreads();
  }
  const mie_step_desc& d = ps_s.d;
  // layer 0's q / k / v rows, out_proj rows, router and norm weights depend on
  // the CTA alone, not on the step's state: staged before the wait
  if (threadIdx.x < 32) att_issue_rows<W>(P, 0);
  if (threadIdx.x == 64) side_issue<W>(P, 0);
  // the previous step's writes (token, position, cache, exchange words, step
  // header) are visible from here on
  pdl_wait();
  // ---- step prologue: position, token, cache slot of the new token; the
  // state words are loaded together (one round trip), the block ids of this
  // CTA's old tokens alongside the new token's block ----
  if (threadIdx.x == 0) {
    const int c = blockIdx.x;
    const int done_v = d.done ? __ldcg(d.done) : 0;
    const int lc = d.log_count ? __ldcg(d.log_count) : 0;
    const int lim = d.step_limit ? __ldcg(d.step_limit) : 0;
    const uint64_t hstep = ll_ld(ps_s.g.ll + kHdrStep);
    const int p = __ldcg(d.pos);
    const int64_t t = __ldcg(d.token);
    int stop = done_v || (d.step_limit && d.log_count && lc >= lim);
    wait_ns_s = d.wait_limit_ns > 0 ? (unsigned long long)d.wait_limit_ns : kWaitLimitNs;
    if (!stop && d.start_gate && !gate_open(d.start_gate, wait_ns_s)) {
      set_status(d.status, MIE_ERR_TIMEOUT);  // the gate stayed closed: the step changes nothing
      stop = 1;
    }
    cx_s.step = (uint32_t)hstep + 1u;
    cx_s.log_k = lc;
    if (!stop && (p < 0 || p >= d.max_pos || t < 0 || t >= d.vocab)) {
      if (c == 0) set_status(d.status, MIE_ERR_RANGE);
      stop = 1;
    }
    int64_t blk = stop ? 0 : p / d.block_size;
    if (!stop && d.block_table) {
      const int pb = __ldcg(d.block_table + blk);
      if (pb < 0 || pb >= d.num_blocks) {
        if (c == 0) set_status(d.status, MIE_ERR_RANGE);
        stop = 1;
      }
      blk = pb;
    }
    cx_s.pos = p;
    cx_s.tok = t;
    cx_s.slot = stop ? 0 : blk * d.kv_stride_block + (int64_t)(p % d.block_size) * d.kv_stride_tok;
    cx_s.blk0 = stop ? 0 : att_split(ps_s.g, d.head_dim, p).t0 / d.block_size;
    cx_s.stop = stop;
  } else if (d.block_table && threadIdx.x <= kStepBlkCache) {
    // physical block ids of this CTA's old tokens, the same for every layer
    // (blk_s[i] by thread i + 1); a position out of range stops the step
    const int p = __ldcg(d.pos), i = threadIdx.x - 1;
    if (p >= 0 && p < d.max_pos) {
      const AttSplit a = att_split(ps_s.g, d.head_dim, p);
      const int b0 = a.t0 / d.block_size;
      if (a.t1 > a.t0 && b0 + i <= (a.t1 - 1) / d.block_size) blk_s[i] = __ldcg(d.block_table + b0 + i);
    }
  }
  __syncthreads();
  if (cx_s.stop) {
    drain_copies();
    return;
  }
  STEP_STAMP(d.num_layers, 4);
  if (threadIdx.x >= 32 && threadIdx.x < 64) att_issue_kv<KV>(P, 0);
  bool ok = true;
#pragma unroll 1
  for (int l = 0; l < d.num_layers && ok; ++l)
    ok = att_phase<W, KV, kWide>(P, l) && proj_phase<W, KV, kWide>(P, l) && moe_phase<W, kWide>(P, l);
  if (ok) ok = head_phase<W, kWide>(P);
  if (!ok) drain_copies();
}

}  // namespace

// ---------------------------------------------------------------------------
// Host side: validation, geometry, launch.
// ---------------------------------------------------------------------------
#ifndef MIE_STEP_WIDE_TU
int step_geometry(const mie_step_desc& d, int grid, StepGeom* g) {
  if (d.num_layers <= 0 || d.num_layers > kMaxStepLayers) return MIE_ERR_UNSUPPORTED;
  if (d.dtype != MIE_F32 && d.dtype != MIE_BF16) return MIE_ERR_UNSUPPORTED;
  if (d.kv_dtype != MIE_F32 && d.kv_dtype != MIE_BF16) return MIE_ERR_UNSUPPORTED;
  const int esz = d.dtype == MIE_BF16 ? 2 : 4, kvsz = d.kv_dtype == MIE_BF16 ? 2 : 4;
  const int D = d.hidden_dim, H = d.num_heads, hd = d.head_dim, Hx = d.expert_hidden_dim, E = d.num_experts;
  if (D <= 0 || H <= 0 || hd <= 0 || Hx <= 0 || H * hd != D || hd % 2) return MIE_ERR_UNSUPPORTED;
  // x lives in one register segment of a warp (at most 768 elements); expert
  // down rows longer than that are multiplied segment by segment (wide)
  if (D > 768 || Hx > kStepMaxExpertHidden || (D * esz) % 16 || (Hx * esz) % 16) return MIE_ERR_UNSUPPORTED;
  // head_dim: whole 16-byte K/V pieces
  if (hd > 128 || (hd * kvsz) % 16) return MIE_ERR_UNSUPPORTED;
  // The narrow geometry: a power-of-two count of K/V pieces per head row,
  // whole PV groups of the CTA's threads, expert rows of one register segment
  // (and for bf16 weights every q row and the selected experts' rows staged in
  // shared memory, checked below).  Other shapes run the wide kernel variant.
  const int vph = hd * kvsz / 16;
  bool wide = (vph & (vph - 1)) != 0 || kStepThreads % hd != 0 || Hx > 768;
  if (d.top_k != 2 || E < 2 || E > 32) return MIE_ERR_UNSUPPORTED;
  if (d.act != MIE_ACT_GELU && d.act != MIE_ACT_SWIGLU) return MIE_ERR_UNSUPPORTED;
  if (d.moe_partial || (d.expert_count && d.expert_count != E) || d.expert_base ||
      (d.moe_peer && d.moe_peer->world > 1) || d.expert_bits)
    return MIE_ERR_UNSUPPORTED;  // expert parallel: the cluster step or layer by layer
  if (d.kv_stride_tok != hd || (d.kv_stride_block * kvsz) % 16 || (d.kv_stride_head * kvsz) % 16)
    return MIE_ERR_UNSUPPORTED;
  if (grid < H || grid < 2) return MIE_ERR_UNSUPPORTED;
  // work splits use 32-bit products (total * grid < 2^32)
  if ((int64_t)d.vocab * grid >= (1ll << 32) || (int64_t)d.max_pos * grid >= (1ll << 32)) return MIE_ERR_UNSUPPORTED;
  if (d.lm_grid < grid) return MIE_ERR_INVALID;  // per-CTA argmax results
  if (d.sample_temperature > 0.f) {  // device sampler
    if (!d.sample_seed || d.sample_top_k > kStepTopKMax) return MIE_ERR_UNSUPPORTED;
    if (d.sample_top_k > 0 && ((d.vocab + grid - 1) / grid > kStepHeadRowsMax || 2 * d.expert_hidden_dim < kStepHeadRowsMax))
      return MIE_ERR_UNSUPPORTED;  // the CTA's logits live in the h vector's shared memory
  }
  StepGeom& G = *g;
  G = StepGeom{};
  G.G = grid;
  G.S = grid / H;
  G.natt = G.S * H;
  // exchange buffers (64-bit words), two copies each
  int64_t off = 8;  // header
  auto take = [&](int64_t words) {
    const int64_t at = off;
    off += (words + 1) & ~int64_t(1);
    return at;
  };
  for (int p = 0; p < 2; ++p) {
    G.off_a[p] = take(D);
    G.off_b[p] = take((int64_t)H * G.S * (3 + hd));
    G.off_c[p] = take(D);
    G.off_d[p] = take(D);
    G.off_e[p] = take(2 * (int64_t)Hx);
  }
  G.off_cand = take((int64_t)grid * kStepTopKMax);
  G.words = off;
  // work per CTA (upper bounds)
  const int kvw_max = 2 * ((hd / 2 + G.S - 1) / G.S) + (hd + G.S - 1) / G.S;  // k + v rows of one split
  const int merge_words = 3 * G.S + G.S * ((hd + G.S - 1) / G.S);
  G.nr_max = (D + grid - 1) / grid;
  const int nu_max = (2 * Hx + grid - 1) / grid;
  const int nmat = d.act == MIE_ACT_SWIGLU ? 2 : 1;
  // per-thread epilogues and the merge gather index table hold one item per thread
  if (merge_words > kStepThreads || 2 * G.nr_max > kStepThreads || nmat * nu_max > kStepThreads ||
      kvw_max > 128 || hd > 128)
    return MIE_ERR_UNSUPPORTED;
  // out_proj rows of a CTA: one per warp of the PROJ threads
  if (G.nr_max > kProjThreads / 32) return MIE_ERR_UNSUPPORTED;
  // shared memory: vectors, then the staging areas
  const uint32_t rbD = (uint32_t)(D * esz), rbH = (uint32_t)(Hx * esz);
  uint32_t so = 0;
  auto stake = [&](uint32_t bytes) {
    so = (so + 127) & ~127u;
    const uint32_t at = so;
    so += bytes;
    return at;
  };
  G.sm_x = stake(4 * D);
  G.sm_xn = stake(4 * D);
  G.sm_xm = stake(4 * D);
  G.sm_h = stake(8 * Hx);
  G.sm_o = stake(4 * D);
  G.sm_qk = stake(4 * (hd + kvw_max));
  int abw = kStepThreads;
  if (E > abw) abw = E;
  G.sm_acc = stake(4 * abw);
  G.chunk_tok = (int)(kStepKvChunkBytes / (2 * hd * kvsz));
  G.sm_sc = stake(4 * G.chunk_tok);
  if (G.S > G.chunk_tok) return MIE_ERR_UNSUPPORTED;  // the merge's split weights live in the scores scratch
  G.sm_anw = stake(2 * rbD);
  const uint32_t base = (so + 127) & ~127u;
  const uint32_t chunk_bytes = (uint32_t)(2 * G.chunk_tok * hd * kvsz);
  const uint32_t att_min = (uint32_t)kvw_max * rbD + chunk_bytes + 3 * 128;
  const uint32_t side_bytes = (uint32_t)(G.nr_max + E + 2) * rbD;
  const uint32_t moe_bytes = (uint32_t)(nmat * nu_max) * rbD + 2u * G.nr_max * rbH;
  // bf16 weights, narrow: the selected experts' rows are staged in shared
  // memory beside every q row of the head.  Wide (and fp32 weights): the
  // expert GEMVs read their rows from global memory (after an L2 prefetch in
  // the wide variant) and as many q rows as fit are staged, the rest read
  // from L2 likewise.
  const uint32_t moe_region = moe_bytes > side_bytes ? moe_bytes : side_bytes;
  if (esz == 2 && base + att_min + moe_region + (uint32_t)hd * rbD > kStepMaxSmem) wide = true;
  G.wide = wide ? 1 : 0;
  // the CTA's LM-head bias values fit in the h vector's shared memory
  G.head_bias_smem = (d.vocab + grid - 1) / grid <= 2 * Hx ? 1 : 0;
  G.moe_staged = esz == 2 && !wide ? 1 : 0;
  const uint32_t region2 = G.moe_staged ? moe_region : side_bytes;
  if (base + att_min + region2 > kStepMaxSmem) return MIE_ERR_UNSUPPORTED;
  const uint32_t avail = kStepMaxSmem - base - region2 - att_min;
  const uint32_t q = avail / rbD;
  G.q_stage = q < (uint32_t)hd ? (int)q : hd;
  G.sm_qw = stake((uint32_t)G.q_stage * rbD);
  G.sm_kvw = stake((uint32_t)kvw_max * rbD);
  G.sm_kv = stake(chunk_bytes);
  const uint32_t att_bytes = G.sm_kv + chunk_bytes - G.sm_qw;
  G.sm_moe = stake(region2);
  G.smem = (so + 127) & ~127u;
  if (G.smem > kStepMaxSmem) return MIE_ERR_UNSUPPORTED;
  // two rows per warp per stage when three such stages fit, else one
  // LM-head ring over [sm_qw, end): the largest stage of 4, 2 or 1 rows per
  // warp that still gives two stages; the first head_early stages lie in the
  // attention area and can be requested before the last layer's MoE is done
  const uint32_t ring_bytes = G.smem - G.sm_qw;
  G.head_rows = 4 * (kStepThreads / 32);
  // the wide variant also has stages of three rows per warp (bf16)
  if (wide && esz == 2 && ring_bytes / ((uint32_t)G.head_rows * rbD) < 2) G.head_rows = 3 * (kStepThreads / 32);
  while (G.head_rows > kStepThreads / 32 && ring_bytes / ((uint32_t)G.head_rows * rbD) < 2) G.head_rows /= 2;
  const uint32_t stage_bytes = (uint32_t)G.head_rows * rbD;
  G.head_stages = (int)(ring_bytes / stage_bytes);
  if (G.head_stages > kStepHeadStagesMax) G.head_stages = kStepHeadStagesMax;
  if (G.head_stages < 2) return MIE_ERR_UNSUPPORTED;
  G.head_early = (int)(att_bytes / stage_bytes);
  // the top-k sampler sorts the candidates of every CTA in the ring area
  if (d.sample_temperature > 0.f && d.sample_top_k > 0) {
    uint32_t n2 = 1;
    while (n2 < (uint32_t)(grid * d.sample_top_k) || n2 < (uint32_t)kStepHeadRowsMax) n2 <<= 1;
    if ((uint64_t)n2 * 8u > ring_bytes) return MIE_ERR_UNSUPPORTED;
  }
  if (G.head_early > G.head_stages) G.head_early = G.head_stages;
  return MIE_OK;
}

int step_launch(const mie_step_desc& d, const StepGeom& g, uint64_t* scratch, cudaStream_t st) {
  StepParams p;
  p.d = d;
  p.g = g;
  p.g.ll = scratch;
  for (int l = 0; l < d.num_layers; ++l) p.layers[l] = d.layers[l];
  p.d.layers = nullptr;
  void (*k)(const StepParams);
#ifdef MIE_STEP_STAMPS
  if (d.num_layers + 1 > kStampLayers || g.G > 160) return MIE_ERR_UNSUPPORTED;
#endif
  if (g.wide) return step_launch_wide(p, st);
  using bf16 = __nv_bfloat16;
  if (d.dtype == MIE_BF16)
    k = d.kv_dtype == MIE_BF16 ? step_kernel<bf16, bf16, false> : step_kernel<bf16, float, false>;
  else
    k = d.kv_dtype == MIE_BF16 ? step_kernel<float, bf16, false> : step_kernel<float, float, false>;
  return launch(k, dim3(g.G), dim3(kStepThreads), g.smem, st, d.use_pdl != 0, p);
}

#ifdef MIE_STEP_STAMPS
// Copy the phase timestamps of the last step to the host (analysis builds).
extern "C" int mie_debug_step_stamps(unsigned long long* host, int64_t count) {
  return cudaMemcpyFromSymbol(host, g_step_stamps, sizeof(unsigned long long) * (size_t)count) == cudaSuccess
             ? MIE_OK
             : MIE_ERR_CUDA;
}
#endif

void step_set_attributes() {
  using bf16 = __nv_bfloat16;
  set_max_smem(step_kernel<bf16, bf16, false>);
  set_max_smem(step_kernel<bf16, float, false>);
  set_max_smem(step_kernel<float, bf16, false>);
  set_max_smem(step_kernel<float, float, false>);
  step_set_attributes_wide();
}

#else
// The wide kernel variant is compiled in its own translation unit
// (step_wide.cu includes this file with MIE_STEP_WIDE_TU defined): sharing
// the out-of-line device functions with it would change their register
// allocation in the narrow variant.
int step_launch_wide(const StepParams& p, cudaStream_t st) {
  void (*k)(const StepParams);
  using bf16 = __nv_bfloat16;
  if (p.d.dtype == MIE_BF16)
    k = p.d.kv_dtype == MIE_BF16 ? step_kernel<bf16, bf16, true> : step_kernel<bf16, float, true>;
  else
    k = p.d.kv_dtype == MIE_BF16 ? step_kernel<float, bf16, true> : step_kernel<float, float, true>;
  return launch(k, dim3(p.g.G), dim3(kStepThreads), p.g.smem, st, p.d.use_pdl != 0, p);
}

void step_set_attributes_wide() {
  using bf16 = __nv_bfloat16;
  set_max_smem(step_kernel<bf16, bf16, true>);
  set_max_smem(step_kernel<bf16, float, true>);
  set_max_smem(step_kernel<float, bf16, true>);
  set_max_smem(step_kernel<float, float, true>);
}

#ifdef MIE_STEP_STAMPS
extern "C" int mie_debug_step_stamps_wide(unsigned long long* host, int64_t count) {
  return cudaMemcpyFromSymbol(host, g_step_stamps, sizeof(unsigned long long) * (size_t)count) == cudaSuccess
             ? MIE_OK
             : MIE_ERR_CUDA;
}
#endif

#endif  // MIE_STEP_WIDE_TU

}  // namespace mie
