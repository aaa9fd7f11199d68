// Expert-parallel all-reduce over peer memory (sm_100a, NVLink / NVSwitch).
//
// The reference is a single-GPU engine; this replaces the NCCL all-reduce of
// the per-layer MoE partial in the expert-parallel decode (the op being split
// is src/moe_engine/fused_moe.py:312-380).  At a [768] fp32 partial the NCCL
// call is all latency (the same ~20 us for fp32 and bf16 on two B200s), so
// this is a one-CTA kernel that moves the partial with plain stores into the
// peers' memory and polls its own:
//
//   tag = seq + 1                       (seq: this group's call counter)
//   for every rank r:  bufs[r][half][rank][i] = {in[i], tag}    (64-bit store)
//   for r = 0 .. world-1:  poll own bufs[rank][half][r][i] until its tag is
//                          `tag`, out[i] += value               (rank order)
//   seq = tag
//
// half = tag & 1.  A rank writes call k + 2's words into half k & 1 only after
// finishing call k + 1, which needed every rank's call k + 1 words, which each
// rank writes only after finishing call k: no word is overwritten before it is
// read.  Every wait is bounded; a rank whose wait ran out records
// MIE_ERR_TIMEOUT and still advances its counter (the group is then broken and
// the caller tears it down).  The receive buffers are plain device
// allocations shared between the rank processes with CUDA IPC.
#include "common.cuh"
#include "exchange.cuh"
#include "kernels.h"

namespace mie {
namespace {

constexpr int kPeerThreads = 1024;

__global__ void __launch_bounds__(kPeerThreads) peer_reduce_kernel(const mie_peer_reduce_args a) {
  __shared__ uint32_t tag_s;
  const int i = threadIdx.x, n = a.n, world = a.world, rank = a.rank;
  if (i == 0) tag_s = *reinterpret_cast<volatile uint32_t*>(a.seq) + 1u;
  __syncthreads();
  const uint32_t tag = tag_s;
  const size_t half = (size_t)(tag & 1u) * (size_t)world * n;
  const unsigned long long limit = a.wait_limit_ns > 0 ? (unsigned long long)a.wait_limit_ns : kWaitLimitNs;
  bool late = false;
  if (i < n) {
    const float v = a.in[i];
    // this rank's slot in every rank's buffer (its own included)
    for (int r = 0; r < world; ++r) ll_put_sys(a.bufs[r] + half + (size_t)rank * n + i, v, tag);
    const uint64_t* mine = a.bufs[rank] + half + i;
    float sum = 0.f;
    for (int r = 0; r < world && !late; ++r) {
      const uint64_t* p = mine + (size_t)r * n;
      uint64_t w = ll_ld_sys(p);
      if (ll_tag(w) != tag) {
        const unsigned long long t0 = global_ns();
        while (ll_tag(w = ll_ld_sys(p)) != tag) {
          if (global_ns() - t0 > limit) {
            late = true;
            break;
          }
        }
      }
      if (!late) sum += ll_val(w);
    }
    a.out[i] = sum;
  }
  if (__syncthreads_or(late) && i == 0) set_status(a.status, MIE_ERR_TIMEOUT);
  if (i == 0) *reinterpret_cast<volatile uint32_t*>(a.seq) = tag;
}

}  // namespace

int64_t peer_buffer_bytes(int n, int world) { return (int64_t)2 * world * n * (int64_t)sizeof(uint64_t); }

int peer_reduce(const mie_peer_reduce_args& a, cudaStream_t st) {
  if (a.n < 1 || a.n > kPeerThreads || a.world < 1 || a.world > MIE_PEER_MAX_RANKS || a.rank < 0 ||
      a.rank >= a.world || !a.in || !a.out || !a.seq)
    return MIE_ERR_INVALID;
  for (int r = 0; r < a.world; ++r)
    if (!a.bufs[r] || (reinterpret_cast<uintptr_t>(a.bufs[r]) & 7u)) return MIE_ERR_INVALID;
  const int threads = (a.n + 31) / 32 * 32;
  return launch(peer_reduce_kernel, dim3(1), dim3(threads), 0, st, false, a);
}

}  // namespace mie
