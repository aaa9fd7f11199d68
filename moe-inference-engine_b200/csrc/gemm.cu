// Tensor-core GEMM for the prompt prefill: C = A . B^T with A [M, K] and
// B [N, K] bf16, both K-major (row-major rows of K elements), on the
// 5th-generation tensor cores.  At a prompt of a few hundred tokens every
// projection of a layer is an M = T problem where tensor cores matter (the
// decode step, M = 1, stays on CUDA cores).
//
// One CTA computes one 128 x BN tile:
//   warp 0      one thread streams K-slices of A and B into shared memory with
//               tiled TMA loads (128-byte swizzle), a ring of kStages stages;
//   warp 1      allocates the TMEM accumulator (BN fp32 columns x 128 lanes)
//               and one thread issues tcgen05.mma (M 128, N BN, K 16) four
//               times per 64-wide K-slice, releasing each stage with
//               tcgen05.commit to the stage's "empty" mbarrier;
//   warps 2-5   wait for the final commit, read the accumulator with
//               tcgen05.ld (warp w reads TMEM lanes 32 (w % 4) ...) and apply
//               the epilogue: optional per-column bias, then fp32 / bf16
//               store, fp32 residual add, GELU (erf), or SwiGLU of a gate half
//               and an up half of the tile.
// Grouped mode (blockIdx.z = group, e.g. an expert): A, B and C rows are
// offset by a per-group stride and rows at or past the group's count (read on
// the device) are neither computed into C nor stored.
//
// Every wait is bounded (kWaitLimitNs); a CTA that gives up records
// MIE_ERR_TIMEOUT, skips its remaining work and still frees its TMEM.
#include <cuda.h>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace mie {
namespace {

constexpr int kGemmThreads = 192;  // 6 warps
constexpr int kBM = 128, kBK = 64;
constexpr int kStages = 4;
constexpr uint32_t kTileABytes = kBM * kBK * 2;  // 16 KB

// ---- tcgen05 / TMA primitives ----
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }
__device__ __forceinline__ float gelu_f(float v) { return 0.5f * v * (1.0f + erff(v * 0.7071067811865476f)); }

template <int BN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const __grid_constant__ CUtensorMap map_b2, const GemmArgs args) {
  constexpr uint32_t kTileBBytes = (uint32_t)BN * kBK * 2;
  constexpr uint32_t kStageBytes = kTileABytes + kTileBBytes;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kStages], empty_bar[kStages], acc_bar;
  __shared__ uint32_t tmem_s;
  __shared__ int bad_s;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.z;
  const int rows = args.counts ? min(__ldg(args.counts + g), args.M) : args.M;
  const int m0 = blockIdx.x * kBM, n0 = blockIdx.y * BN;
  if (m0 >= rows) return;  // whole CTA: past this group's rows
  const int a_row0 = g * args.a_group_rows + m0;
  const int b_row0 = g * args.b_group_rows + (EPI == kEpiSwiGLU ? n0 / 2 : n0);
  const int nk = args.K / kBK;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&acc_bar, 1);
    bad_s = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&tmem_s, (uint32_t)BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_s;

  if (warp == 0 && lane == 0) {
    // ---- TMA producer ----
    for (int k = 0; k < nk; ++k) {
      const int s = k % kStages, use = k / kStages;
      if (use > 0 && !mbar_wait(&empty_bar[s], (uint32_t)((use - 1) & 1), args.status)) {
        bad_s = 1;
        break;
      }
      uint8_t* sa = smem + (size_t)s * kStageBytes;
      uint8_t* sb = sa + kTileABytes;
      mbar_arrive_expect_tx(&full_bar[s], kStageBytes);
      tma_load_2d(sa, &map_a, k * kBK, a_row0, &full_bar[s]);
      if constexpr (EPI == kEpiSwiGLU) {
        // gate rows then up rows of the same BN / 2 units
        tma_load_2d(sb, &map_b, k * kBK, b_row0, &full_bar[s]);
        tma_load_2d(sb + kTileBBytes / 2, &map_b2, k * kBK, b_row0, &full_bar[s]);
      } else {
        tma_load_2d(sb, &map_b, k * kBK, b_row0, &full_bar[s]);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    constexpr uint32_t idesc = idesc_bf16(BN);
    bool ok = true;
    for (int k = 0; k < nk && ok; ++k) {
      const int s = k % kStages, use = k / kStages;
      if (!mbar_wait(&full_bar[s], (uint32_t)(use & 1), args.status)) {
        bad_s = 1;
        ok = false;
        break;
      }
      tc_fence_after();
      const uint8_t* sa = smem + (size_t)s * kStageBytes;
      const uint8_t* sb = sa + kTileABytes;
#pragma unroll
      for (int kk = 0; kk < kBK / 16; ++kk)
        tc_mma(tmem, sw128_desc(sa, 32u * kk), sw128_desc(sb, 32u * kk), idesc, (k | kk) ? 1u : 0u);
      tc_commit(&empty_bar[s]);  // the stage is free once these MMAs have read it
    }
    tc_commit(&acc_bar);  // accumulator complete (also after a failed wait: nothing in flight is left)
  } else if (warp >= 2) {
    // ---- epilogue: TMEM lanes 32 q .. 32 q + 31 = tile rows ----
    const int q = warp & 3;
    const bool ok = mbar_wait(&acc_bar, 0u, args.status);
    tc_fence_after();
    const int r = q * 32 + lane;
    const int row = m0 + r;
    const int64_t crow = (int64_t)g * args.c_group_rows + row;
    if (ok && !bad_s) {
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16);
      if constexpr (EPI == kEpiSwiGLU) {
        // columns [0, BN/2): gate, [BN/2, BN): up of the same units
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 32) {
          float gv[32], uv[32];
          tmem_ld32(tbase + c, gv);
          tmem_ld32(tbase + BN / 2 + c, uv);
          if (row < rows) {
            __nv_bfloat16* out = static_cast<__nv_bfloat16*>(args.c) + crow * args.ldc + n0 / 2 + c;
#pragma unroll
            for (int i = 0; i < 32; i += 2)
              *reinterpret_cast<__nv_bfloat162*>(out + i) =
                  __floats2bfloat162_rn(silu_f(gv[i]) * uv[i], silu_f(gv[i + 1]) * uv[i + 1]);
          }
        }
      } else {
        const __nv_bfloat16* bias = args.bias ? args.bias + (int64_t)g * args.bias_group_stride + n0 : nullptr;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          float v[32];
          tmem_ld32(tbase + c, v);
          if (bias) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] += __bfloat162float(bias[c + i]);
          }
          if (row < rows) {
            if constexpr (EPI == kEpiBF16 || EPI == kEpiGelu) {
              if constexpr (EPI == kEpiGelu) {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = gelu_f(v[i]);
              }
              __nv_bfloat16* out = static_cast<__nv_bfloat16*>(args.c) + crow * args.ldc + n0 + c;
#pragma unroll
              for (int i = 0; i < 32; i += 2)
                *reinterpret_cast<__nv_bfloat162*>(out + i) = __floats2bfloat162_rn(v[i], v[i + 1]);
            } else {
              float* out = static_cast<float*>(args.c) + crow * args.ldc + n0 + c;
              if constexpr (EPI == kEpiResid) {
                const float* res = args.resid + crow * args.ldr + n0 + c;
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                  const float4 rv = *reinterpret_cast<const float4*>(res + i);
                  *reinterpret_cast<float4*>(out + i) =
                      make_float4(rv.x + v[i], rv.y + v[i + 1], rv.z + v[i + 2], rv.w + v[i + 3]);
                }
              } else {
#pragma unroll
                for (int i = 0; i < 32; i += 4)
                  *reinterpret_cast<float4*>(out + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
              }
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_free(tmem, (uint32_t)BN);
  }
}

// ---- host: tensor maps ----
}  // namespace

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

namespace {

// 2-D bf16 tensor [rows, cols] (row stride ld elements), box box_rows x 64,
// 128-byte swizzle; reads past `rows` return zeros.
int make_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return MIE_ERR_CUDA;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MIE_OK : MIE_ERR_INVALID;
}

template <int BN, int EPI>
constexpr uint32_t gemm_smem() {
  return 1024 + kStages * (kTileABytes + (uint32_t)BN * kBK * 2);
}

template <int BN, int EPI>
int gemm_launch_t(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& b2, const GemmArgs& args,
                  int groups, cudaStream_t st) {
  const dim3 grid((unsigned)((args.M + kBM - 1) / kBM), (unsigned)(args.N / BN), (unsigned)groups);
  return launch(gemm_kernel<BN, EPI>, grid, dim3(kGemmThreads), gemm_smem<BN, EPI>(), st, false, a, b, b2, args);
}

}  // namespace

void gemm_set_attributes() {
  cudaFuncSetAttribute(gemm_kernel<128, kEpiF32>, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm_smem<128, kEpiF32>());
  cudaFuncSetAttribute(gemm_kernel<128, kEpiBF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       gemm_smem<128, kEpiBF16>());
  cudaFuncSetAttribute(gemm_kernel<128, kEpiResid>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       gemm_smem<128, kEpiResid>());
  cudaFuncSetAttribute(gemm_kernel<128, kEpiSwiGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       gemm_smem<128, kEpiSwiGLU>());
  cudaFuncSetAttribute(gemm_kernel<128, kEpiGelu>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       gemm_smem<128, kEpiGelu>());
}

// C[g] = A[g] . B[g]^T for the groups of a (see mie_gemm_args).
int gemm_run(const mie_gemm_args& a, cudaStream_t st) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0 || a.K % kBK || a.N % 128 || a.groups <= 0) return MIE_ERR_UNSUPPORTED;
  if (!a.a || !a.b || !a.c || (a.epilogue == kEpiSwiGLU && (!a.b2 || a.bias)) ||
      (a.epilogue == kEpiResid && !a.resid) || a.epilogue < kEpiF32 || a.epilogue > kEpiGelu)
    return MIE_ERR_INVALID;
  const bool grouped = a.groups > 1 || a.counts;
  if (grouped && (a.a_group_rows < a.M || a.c_group_rows < a.M)) return MIE_ERR_INVALID;
  const uintptr_t al = reinterpret_cast<uintptr_t>(a.a) | reinterpret_cast<uintptr_t>(a.b) |
                       reinterpret_cast<uintptr_t>(a.b2) | (uintptr_t)(a.lda * 2) | (uintptr_t)(a.ldb * 2);
  if (al % 16 || a.lda < a.K || a.ldb < a.K) return MIE_ERR_INVALID;
  const int out_cols = a.epilogue == kEpiSwiGLU ? a.N / 2 : a.N;
  if (a.ldc < out_cols || (a.epilogue == kEpiResid && a.ldr < a.N)) return MIE_ERR_INVALID;
  // epilogue stores: 16-byte fp32 vectors, 4-byte bf16 pairs
  const bool f32_out = a.epilogue == kEpiF32 || a.epilogue == kEpiResid;  // else bf16 out
  const uintptr_t cal = reinterpret_cast<uintptr_t>(a.c) | reinterpret_cast<uintptr_t>(a.resid) |
                        (uintptr_t)(a.ldc * (f32_out ? 4 : 2)) | (uintptr_t)(a.ldr * 4);
  if (cal % (f32_out ? 16 : 4)) return MIE_ERR_INVALID;
  const int64_t a_rows = grouped ? (int64_t)a.groups * a.a_group_rows : a.M;
  CUtensorMap ma, mb, mb2;
  const int box_b = a.epilogue == kEpiSwiGLU ? 64 : 128;
  int rc = make_map(&ma, a.a, a_rows, a.K, a.lda, kBM);
  if (rc == MIE_OK) rc = make_map(&mb, a.b, a.b_rows, a.K, a.ldb, box_b);
  if (rc == MIE_OK) rc = make_map(&mb2, a.epilogue == kEpiSwiGLU ? a.b2 : a.b, a.b_rows, a.K, a.ldb, box_b);
  if (rc != MIE_OK) return rc;
  GemmArgs g{};
  g.M = a.M;
  g.N = a.N;
  g.K = a.K;
  g.c = a.c;
  g.ldc = a.ldc;
  g.resid = a.resid;
  g.ldr = a.ldr;
  g.counts = a.counts;
  g.a_group_rows = grouped ? a.a_group_rows : 0;
  g.b_group_rows = grouped ? a.b_group_rows : 0;
  g.c_group_rows = grouped ? a.c_group_rows : 0;
  g.status = a.status;
  g.bias = static_cast<const __nv_bfloat16*>(a.bias);
  g.bias_group_stride = grouped ? a.bias_group_stride : 0;
  switch (a.epilogue) {
    case kEpiF32:
      return gemm_launch_t<128, kEpiF32>(ma, mb, mb2, g, a.groups, st);
    case kEpiBF16:
      return gemm_launch_t<128, kEpiBF16>(ma, mb, mb2, g, a.groups, st);
    case kEpiResid:
      return gemm_launch_t<128, kEpiResid>(ma, mb, mb2, g, a.groups, st);
    case kEpiGelu:
      return gemm_launch_t<128, kEpiGelu>(ma, mb, mb2, g, a.groups, st);
    default:
      return gemm_launch_t<128, kEpiSwiGLU>(ma, mb, mb2, g, a.groups, st);
  }
}

}  // namespace mie
