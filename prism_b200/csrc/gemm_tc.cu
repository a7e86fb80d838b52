// Dense GEMM on the sm_100a tensor cores for the self-attention layer's
// projections (q / k / v / o: F.linear in SelfAttention.forward,
// hymm/models/modules/wan_video_dit.py:699-701, 841) and their backward:
//
//   C[M, N] (bf16, row stride ldc) (+)= sum_k A(m, k) B(n, k)  (+ bias[n], fp32 accumulation)
//
// Each operand is a bf16 row-major tensor that is either K-major (K contiguous:
// A(m, k) = A[m * lda + k]) or MN-major (M or N contiguous: A(m, k) = A[k * lda + m]):
//   forward  y  = x W^T  : A = x  [M, K] K-major,  B = W [N, K] K-major
//   dgrad    dx = dy W   : A = dy [M, N] K-major,  B = W  MN-major
//   wgrad    dW = dy^T x : A = dy   MN-major,      B = x  MN-major
//
// Persistent kernel, one CTA per SM: 128 x 256 output tiles, K in steps of 64.
// Warp 4 streams A / B tiles with TMA (128B swizzle) into a 4-stage ring, warp 5
// issues tcgen05.mma (M = 128, N = 256, K = 16; A and B from shared memory) into
// one of two TMEM accumulators (2 x 256 columns), so the epilogue warps 0-3
// (thread = output row) drain tile t while the tensor core computes tile t + 1.
// Per K = 16 the MMA reads 4 KB of A and 8 KB of B in 128 clocks (96 B/clk of the
// 128 B/clk shared-memory port), leaving room for the TMA fills.  Every wait is
// bounded (sm100.cuh); a wait that gives up sets the GEMM's device error word.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include <mutex>

#include "prism_common.cuh"
#include "sm100.cuh"

namespace prism {
namespace gemm {

using namespace sm100;

__device__ int g_gemm_error = 0;
enum : int { kErrProducer = 401, kErrMma = 402, kErrEpilogue = 403 };

constexpr int kThreads = 192;
constexpr int kStages = 4;
constexpr int kTileM = 128, kTileN = 256, kTileK = 64;
constexpr int kABytes = kTileM * kTileK * 2, kBBytes = kTileN * kTileK * 2;  // 16 KB, 32 KB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int B_FULL = 0, B_EMPTY = kStages, B_ACC_FULL = 2 * kStages, B_ACC_EMPTY = B_ACC_FULL + 2,
              B_DRAIN = B_ACC_EMPTY + 2, NBAR = B_DRAIN + 1;
constexpr int SM_BAR = kStages * kStageBytes;
constexpr int SM_TMEM = SM_BAR + NBAR * 8;
constexpr int SM_ABORT = SM_TMEM + 4;
constexpr size_t kSmemBytes = 1024 + SM_ABORT + 4;

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~(uintptr_t)1023);
}

// Four K = 16 MMAs of one K = 64 stage: descriptor steps in 16-byte units, 32 B
// inside a K-major 128-byte row, 2048 B (16 rows) for an MN-major operand.
template <bool kAMn, bool kBMn>
__device__ __forceinline__ void mma_stage(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                          uint32_t accumulate) {
  if constexpr (!kAMn && !kBMn) mma_chain4<2, 4, 6, 2, 4, 6>(d_tmem, a, b, idesc, accumulate);
  else if constexpr (!kAMn && kBMn) mma_chain4<2, 4, 6, 128, 256, 384>(d_tmem, a, b, idesc, accumulate);
  else if constexpr (kAMn && !kBMn) mma_chain4<128, 256, 384, 2, 4, 6>(d_tmem, a, b, idesc, accumulate);
  else mma_chain4<128, 256, 384, 128, 256, 384>(d_tmem, a, b, idesc, accumulate);
}

template <bool kAMn, bool kBMn>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                   int M, int N, int K, const float* __restrict__ bias, __nv_bfloat16* __restrict__ c,
                   int64_t ldc, int accumulate) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  const uint32_t sb = smem_u32(sm);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto bar = [&](int i) { return sb + SM_BAR + 8 * i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + SM_ABORT);
  const int tm = (M + kTileM - 1) / kTileM, tn = (N + kTileN - 1) / kTileN;
  const int tiles = tm * tn, nk = (K + kTileK - 1) / kTileK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(bar(B_FULL + i), 1);
      mbar_init(bar(B_EMPTY + i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(B_ACC_FULL + i), 1);
      mbar_init(bar(B_ACC_EMPTY + i), 4);
    }
    mbar_init(bar(B_DRAIN), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(sb + SM_TMEM, 512);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + SM_TMEM);

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
        const int m0 = (t / tn) * kTileM, n0 = (t % tn) * kTileN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % kStages;
          if (it >= kStages &&
              !mbar_wait(bar(B_EMPTY + s), ((it / kStages) - 1) & 1, abort_flag, &g_gemm_error, kErrProducer)) {
            ok = false;
            break;
          }
          const uint32_t a_dst = sb + s * kStageBytes, b_dst = a_dst + kABytes, fb = bar(B_FULL + s);
          mbar_expect_tx(fb, kStageBytes);
          const int k0 = kb * kTileK;
          if constexpr (!kAMn) {
            tma_load_2d(a_dst, &tm_a, k0, m0, fb);                 // box {64 K, 128 M}
          } else {
#pragma unroll
            for (int j = 0; j < kTileM / 64; ++j)                  // box {64 M, 64 K} per 64 columns
              tma_load_2d(a_dst + j * 8192, &tm_a, m0 + 64 * j, k0, fb);
          }
          if constexpr (!kBMn) {
            tma_load_2d(b_dst, &tm_b, k0, n0, fb);                 // box {64 K, 256 N}
          } else {
#pragma unroll
            for (int j = 0; j < kTileN / 64; ++j)
              tma_load_2d(b_dst + j * 8192, &tm_b, n0 + 64 * j, k0, fb);
          }
        }
      }
      // drain: every issued copy has landed before the CTA may leave
      for (int m = (it > kStages ? it - kStages : 0); m < it; ++m)
        mbar_wait(bar(B_FULL + m % kStages), (m / kStages) & 1, abort_flag, &g_gemm_error, kErrProducer);
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16(kTileM, kTileN, kAMn, kBMn);
      int it = 0, tl = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x, ++tl) {
        const int ab = tl & 1;
        if (tl >= 2 &&
            !mbar_wait(bar(B_ACC_EMPTY + ab), ((tl >> 1) - 1) & 1, abort_flag, &g_gemm_error, kErrMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(bar(B_FULL + s), (it / kStages) & 1, abort_flag, &g_gemm_error, kErrMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_src = sb + s * kStageBytes, b_src = a_src + kABytes;
          const uint64_t da = kAMn ? desc_mn_sw128(a_src, 8192) : desc_k_sw128(a_src);
          const uint64_t db = kBMn ? desc_mn_sw128(b_src, 8192) : desc_k_sw128(b_src);
          mma_stage<kAMn, kBMn>(tmem + ab * kTileN, da, db, IDESC, kb > 0 ? 1u : 0u);
          mma_commit(bar(B_EMPTY + s));
        }
        if (ok) mma_commit(bar(B_ACC_FULL + ab));
      }
      mma_commit(bar(B_DRAIN));
      mbar_wait(bar(B_DRAIN), 0, abort_flag, &g_gemm_error, kErrMma);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const uint32_t t_lane = tmem + ((uint32_t)(warp * 32) << 16);
    int tl = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++tl) {
      const int ab = tl & 1;
      const int m0 = (t / tn) * kTileM, n0 = (t % tn) * kTileN;
      const int row = m0 + warp * 32 + lane;
      bool ok = mbar_wait(bar(B_ACC_FULL + ab), (tl >> 1) & 1, abort_flag, &g_gemm_error, kErrEpilogue);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
#pragma unroll 1
      for (int cc = 0; cc < kTileN / 32; ++cc) {
        const int col0 = n0 + cc * 32;
        uint32_t raw[32];
        tmem_ld32(t_lane + ab * kTileN + cc * 32, raw);
        tmem_wait_ld_dep(raw);
        if (row < M && col0 < N) {
          __nv_bfloat16* dst = c + (int64_t)row * ldc + col0;
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            if (col0 + 8 * g >= N) break;
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              v[i] = __uint_as_float(raw[8 * g + i]);
              if (bias != nullptr) v[i] += __ldg(bias + col0 + 8 * g + i);
            }
            uint4* p = reinterpret_cast<uint4*>(dst + 8 * g);
            if (accumulate) {
              const uint4 o = *p;
              const uint32_t ow[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                v[2 * i] += __uint_as_float(ow[i] << 16);
                v[2 * i + 1] += __uint_as_float(ow[i] & 0xffff0000u);
              }
            }
            *p = make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]),
                            pack_bf16(v[6], v[7]));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_ACC_EMPTY + ab));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ host
using EncodeFn = PFN_cuTensorMapEncodeTiled_v12000;

static EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  return fn;
}

// 2D bf16 map of a row-major [rows, cols] tensor (row stride ld elements), boxes of
// box_cols x box_rows, 128-byte swizzle (box_cols = 64: one 128-byte row).
static prism_status_t make_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int64_t ld,
                               int box_rows) {
  EncodeFn enc = encode_fn();
  if (enc == nullptr) {
    set_error("prism_gemm: cuTensorMapEncodeTiled is unavailable from the driver");
    return PRISM_ERR_CUDA;
  }
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("prism_gemm: cuTensorMapEncodeTiled failed (%d)", (int)r);
    return PRISM_ERR_CUDA;
  }
  return PRISM_OK;
}

template <bool kAMn, bool kBMn>
static prism_status_t launch(const CUtensorMap& ma, const CUtensorMap& mb, int M, int N, int K,
                             const float* bias, void* c, int64_t ldc, int accumulate, cudaStream_t stream) {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    PRISM_CHECK_CUDA(cudaGetDevice(&dev), "prism_gemm: cudaGetDevice");
    PRISM_CHECK_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev),
                     "prism_gemm: SM count");
  }
  PRISM_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<kAMn, kBMn>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)kSmemBytes),
                   "prism_gemm: smem attribute");
  const int64_t tiles = (int64_t)((M + kTileM - 1) / kTileM) * ((N + kTileN - 1) / kTileN);
  const unsigned grid = (unsigned)(tiles < sms ? tiles : sms);
  gemm_tc_kernel<kAMn, kBMn><<<grid, kThreads, kSmemBytes, stream>>>(ma, mb, M, N, K, bias,
                                                                     (__nv_bfloat16*)c, ldc, accumulate);
  PRISM_CHECK_LAUNCH("prism_gemm");
  return PRISM_OK;
}

}  // namespace gemm
}  // namespace prism

using namespace prism;

int prism_gemm_device_status_internal(void) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, gemm::g_gemm_error, sizeof(int)) != cudaSuccess) return -1;
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(gemm::g_gemm_error, &zero, sizeof(int));
  }
  return v;
}

extern "C" prism_status_t prism_gemm_bf16(const void* a, int64_t lda, int a_mn_major, const void* b,
                                          int64_t ldb, int b_mn_major, int M, int N, int K,
                                          const float* bias, void* c, int64_t ldc, int accumulate,
                                          cudaStream_t stream) {
  PRISM_CHECK_ARG(a && b && c, "prism_gemm: null pointer");
  PRISM_CHECK_ARG(M >= 1 && N >= 1 && K >= 1, "prism_gemm: sizes must be positive");
  PRISM_CHECK_ARG(N % 8 == 0 && ldc % 8 == 0 && ldc >= N && lda % 8 == 0 && ldb % 8 == 0,
                  "prism_gemm: N and the row strides must be multiples of 8 elements");
  PRISM_CHECK_ARG(aligned16(a) && aligned16(b) && aligned16(c), "prism_gemm: tensors must be 16-byte aligned");
  PRISM_CHECK_ARG(a_mn_major ? (lda >= M && M % 8 == 0) : lda >= K, "prism_gemm: bad A stride");
  PRISM_CHECK_ARG(b_mn_major ? (ldb >= N) : ldb >= K, "prism_gemm: bad B stride");
  PRISM_CHECK_ARG(a_mn_major || K % 8 == 0, "prism_gemm: K-major A needs K % 8 == 0");
  PRISM_CHECK_ARG(b_mn_major || K % 8 == 0, "prism_gemm: K-major B needs K % 8 == 0");
  CUtensorMap ma, mb;
  // K-major: [rows = M or N, cols = K], box {64 K, tile rows}; MN-major: [rows = K,
  // cols = M or N], box {64, 64}
  prism_status_t st = a_mn_major ? gemm::make_map(&ma, a, K, M, lda, 64)
                                 : gemm::make_map(&ma, a, M, K, lda, gemm::kTileM);
  if (st != PRISM_OK) return st;
  st = b_mn_major ? gemm::make_map(&mb, b, K, N, ldb, 64) : gemm::make_map(&mb, b, N, K, ldb, gemm::kTileN);
  if (st != PRISM_OK) return st;
  if (!a_mn_major && !b_mn_major) return gemm::launch<false, false>(ma, mb, M, N, K, bias, c, ldc, accumulate, stream);
  if (!a_mn_major && b_mn_major) return gemm::launch<false, true>(ma, mb, M, N, K, bias, c, ldc, accumulate, stream);
  if (a_mn_major && !b_mn_major) return gemm::launch<true, false>(ma, mb, M, N, K, bias, c, ldc, accumulate, stream);
  return gemm::launch<true, true>(ma, mb, M, N, K, bias, c, ldc, accumulate, stream);
}
