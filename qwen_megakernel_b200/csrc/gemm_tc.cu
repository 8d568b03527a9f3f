// Tensor-core GEMM of the token-parallel path (prefill and batched decode) on
// B200: tcgen05.mma with TMEM accumulators, operands staged by TMA
// (cp.async.bulk.tensor, 128-byte swizzle, no multicast) in a multi-stage
// shared-memory ring guarded by mbarriers.
//
//   C[z][split] (fp32, [rows, n], row stride ldc)
//       = A[z][rows, K_split] (bf16, row-major) * W[z][n, K_split]^T (bf16, row-major)
//
// The projections use it with W = a weight matrix [out, in] and A = the
// activations (rows = tokens, fp32 values stacked as a bf16 hi half and a lo
// half, see batch.cu); the prompt attention uses it with W = the K cache
// (scores) and W = the transposed V cache (P V).  All operands are K-major.
//
// One CTA computes a 128 x TN tile of C^T: W rows m0 .. m0+127 are the MMA's
// M = 128 operand (TMEM lane = W row), A rows n0 .. n0+TN-1 the N operand
// (TMEM column = A row).  Warp 0 (one lane) issues the TMA loads of 64-element
// K blocks, warp 1 (one lane) the MMAs (4 of K = 16 per block) and
// tcgen05.commit, which frees a ring stage once its MMAs have read it; then
// all four warps read the accumulator (tcgen05.ld, lane = W row) and store C
// column by column, 32 consecutive W rows per warp store (coalesced).
// Split-K: z = batch * splits + split; split s covers K blocks
// [s * kb_per_split, ...) and writes its own partial C (the consumer adds the
// partials in a fixed order, so results do not depend on timing).
//
// Every wait is bounded (1 s): on expiry the CTA sets QMK_BATCH_TIMEOUT in
// the caller's status word, stops issuing, lets what it issued complete
// (bounded again) and exits without storing.

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>

#include "qmk_device.cuh"
#include "qwen_megakernel.h"

__attribute__((visibility("hidden"))) int qmk_internal_set_error(int code, const char *msg);
__attribute__((visibility("hidden"))) int qmk_internal_clear_error();

namespace qgemm {

using namespace qmk;

constexpr int kBM = 128;                 // W rows per tile (MMA M)
constexpr int kBK = 64;                  // K elements per ring stage (one 128-byte swizzle row)
constexpr int kThreads = 128;
constexpr int kWBytes = kBM * kBK * 2;   // 16 KB
constexpr unsigned long long kWaitNs = 1000000000ull;

struct Args {
  CUtensorMap tw;  // W: dims {K, n, batch}, box {64, 128, 1}
  CUtensorMap ta;  // A: dims {K, rows, batch}, box {64, TN, 1}
  float *C;
  long long ldc, c_batch, c_split;
  int n, rows, kb_total, kb_per_split, splits;
  unsigned *status;
};

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y, int z, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_map(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Bounded mbarrier wait; false on timeout or when the CTA is aborting.
__device__ __forceinline__ bool wait_bar(uint64_t *bar, unsigned parity, volatile int *abort_flag) {
  uint64_t t0 = 0;
  for (unsigned it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 63u) {
      if (*abort_flag) return false;
      const uint64_t now = global_timer_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > kWaitNs) {
        return false;
      }
    }
  }
}

template <int TN>
__host__ __device__ constexpr int tmem_cols() {
  return TN <= 32 ? 32 : TN <= 64 ? 64 : TN <= 128 ? 128 : 256;
}

template <int TN, int STAGES>
__host__ __device__ constexpr int smem_bytes() {
  return STAGES * (kWBytes + TN * kBK * 2) + 1024 /* alignment slack */ + 256 /* barriers */;
}

template <int TN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ Args g) {
  constexpr int kABytes = TN * kBK * 2;
  constexpr int kStageBytes = kWBytes + kABytes;
  constexpr int kCols = tmem_cols<TN>();
  static_assert(TN % 32 == 0 && TN <= 256, "TN: 32 .. 256 in steps of 32");
  static_assert(kStageBytes % 1024 == 0, "stages must keep 1 KB swizzle-atom alignment");
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * kStageBytes);
  uint64_t *empty = full + STAGES;
  uint64_t *acc_bar = empty + STAGES;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_bar + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m0 = blockIdx.x * kBM, n0 = blockIdx.y * TN;
  const int batch = blockIdx.z / g.splits, split = blockIdx.z % g.splits;
  const int kb0 = split * g.kb_per_split;
  const int kb1 = min(g.kb_total, kb0 + g.kb_per_split);
  const int nkb = kb1 - kb0;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_bar, 1);
    fence_mbar_init();
    *abort_flag = 0;
    prefetch_map(&g.tw);
    prefetch_map(&g.ta);
  }
  if (warp == 0) tmem_alloc(tmem_slot, kCols);
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // TMA producer
    int issued = 0;
    for (int i = 0; i < nkb; ++i) {
      const int s = i % STAGES;
      if (i >= STAGES && !wait_bar(&empty[s], ((i / STAGES) - 1) & 1, abort_flag)) {
        *abort_flag = 1;
        break;
      }
      uint8_t *sw = smem + s * kStageBytes;
      mbar_arrive_expect_tx(&full[s], kStageBytes);
      tma_load_3d(sw, &g.tw, (kb0 + i) * kBK, m0, batch, &full[s]);
      tma_load_3d(sw + kWBytes, &g.ta, (kb0 + i) * kBK, n0, batch, &full[s]);
      ++issued;
    }
    // copies in flight must land before the CTA's shared memory goes away
    for (int i = (issued > STAGES ? issued - STAGES : 0); i < issued; ++i) {
      const int s = i % STAGES;
      const uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(&full[s], (i / STAGES) & 1))
        if (global_timer_ns() - t0 > kWaitNs) break;
    }
  } else if (warp == 1) {
    // MMA issuer: the converged warp issues, one elected lane executes
    const uint32_t idesc = mma_idesc_bf16(kBM, TN);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % STAGES;
      bool ok = true;
      if (lane == 0) ok = wait_bar(&full[s], (i / STAGES) & 1, abort_flag);
      if (!__shfl_sync(0xffffffffu, (int)ok, 0)) {
        if (lane == 0) *abort_flag = 1;
        break;
      }
      tc_fence_after_sync();
      const uint8_t *sw = smem + s * kStageBytes;
      const uint64_t ad = smem_desc_sw128(smem_addr(sw), 1024u);
      const uint64_t bd = smem_desc_sw128(smem_addr(sw + kWBytes), 1024u);
#pragma unroll
      for (int kk = 0; kk < kBK / 16; ++kk) tc_mma_bf16_warp(tmem, ad + 2u * kk, bd + 2u * kk, idesc, i > 0 || kk > 0);
      tc_commit_warp(&empty[s]);
    }
    tc_commit_warp(acc_bar);  // completes once every MMA issued above has
  }
  __syncwarp();

  // Epilogue: TMEM lane (32 warp + lane) = W row m0 + 32 warp + lane.  The
  // accumulator commit is waited for even when aborting (bounded by time
  // only): MMAs in flight must finish before TMEM is freed.
  bool ok = true;
  {
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(acc_bar, 0)) {
      if (global_timer_ns() - t0 > kWaitNs) {
        ok = false;
        break;
      }
    }
  }
  ok = ok && *abort_flag == 0 && nkb > 0;
  ok = __all_sync(0xffffffffu, ok);
  if (!ok && lane == 0 && g.status) atomicOr(g.status, QMK_BATCH_TIMEOUT);
  tc_fence_after_sync();
  if (ok) {
    const int m = m0 + 32 * warp + lane;
    float *cb = g.C + (size_t)batch * (size_t)g.c_batch + (size_t)split * (size_t)g.c_split;
#pragma unroll
    for (int c0 = 0; c0 < TN; c0 += 32) {
      uint32_t r[32];
      tmem_ld32(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)c0, r);
      if (m < g.n) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int col = n0 + c0 + j;
          if (col < g.rows) cb[(size_t)col * (size_t)g.ldc + m] = __uint_as_float(r[j]);
        }
      }
    }
  }
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, kCols);
  }
}

// ---------------------------------------------------------------- host side

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
bool g_attr_set[kMaxDevices] = {};

int encode_fn(PFN_cuTensorMapEncodeTiled_v12000 *out) {
  if (!g_encode) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    const cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
      return qmk_internal_set_error(QMK_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  *out = g_encode;
  return QMK_OK;
}

// bf16 [batch][rows][ld] (K = the first `k` elements of a row), box 64 x box_rows.
int make_map(CUtensorMap *m, const void *base, long long k, long long rows, long long ld, long long batch,
             long long batch_stride, int box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  if (encode_fn(&enc) != QMK_OK) return QMK_ERR_CUDA;
  const cuuint64_t dims[3] = {(cuuint64_t)k, (cuuint64_t)rows, (cuuint64_t)batch};
  const cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)(batch > 1 ? batch_stride : rows * ld) * 2};
  const cuuint32_t box[3] = {(cuuint32_t)kBK, (cuuint32_t)box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return qmk_internal_set_error(QMK_ERR_ARGS, "cuTensorMapEncodeTiled rejected an operand");
  return QMK_OK;
}

template <int TN, int STAGES>
int launch(const Args &a, int tiles_m, int tiles_n, int z, cudaStream_t stream, int dev) {
  constexpr int kSmem = smem_bytes<TN, STAGES>();
  static_assert(kSmem <= 232448, "GEMM ring exceeds shared memory");
  cudaError_t e;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    static bool set[kMaxDevices] = {};
    if (!set[dev]) {
      e = cudaFuncSetAttribute(gemm_kernel<TN, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
      if (e != cudaSuccess) return qmk_internal_set_error(QMK_ERR_CUDA, "GEMM kernel shared memory attribute");
      set[dev] = true;
    }
  }
  gemm_kernel<TN, STAGES><<<dim3(tiles_m, tiles_n, z), kThreads, kSmem, stream>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return qmk_internal_set_error(QMK_ERR_CUDA, cudaGetErrorString(e));
  return QMK_OK;
}

}  // namespace qgemm

// Internal entry (batch.cu): see qmk_gemm_bf16_nt in include/qwen_megakernel.h.
__attribute__((visibility("hidden"))) int qmk_internal_gemm(
    const void *W, long long ldw, long long w_batch_stride, int n, const void *A, long long lda,
    long long a_batch_stride, int rows, int k, int batch, int splits, float *C, long long ldc, long long c_batch_stride,
    long long c_split_stride, unsigned *status, cudaStream_t stream) {
  using namespace qgemm;
  if (!W || !A || !C || n < 1 || rows < 1 || k < 1 || batch < 1 || splits < 1)
    return qmk_internal_set_error(QMK_ERR_ARGS, "qmk_gemm: null operand or empty shape");
  if ((reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(A)) % 16 || (ldw | lda) % 8 ||
      (batch > 1 && (w_batch_stride | a_batch_stride) % 8))
    return qmk_internal_set_error(QMK_ERR_ARGS, "qmk_gemm: operands and strides must be 16-byte aligned");
  if (ldw < k || lda < k || ldc < n)
    return qmk_internal_set_error(QMK_ERR_ARGS, "qmk_gemm: leading dimension smaller than the row");
  const int kb_total = (k + kBK - 1) / kBK;
  int kbps = (kb_total + splits - 1) / splits;
  splits = (kb_total + kbps - 1) / kbps;  // no empty split
  if (splits > 1 && (k % kBK))
    return qmk_internal_set_error(QMK_ERR_ARGS, "qmk_gemm: split-K needs K a multiple of 64");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return qmk_internal_set_error(QMK_ERR_CUDA, "qmk_gemm: cudaGetDevice");
  const int tn = rows <= 32 ? 32 : rows <= 64 ? 64 : rows <= 128 ? 128 : 256;
  Args a;
  memset(&a, 0, sizeof(a));
  if (make_map(&a.tw, W, k, n, ldw, batch, w_batch_stride, kBM) != QMK_OK) return QMK_ERR_ARGS;
  if (make_map(&a.ta, A, k, rows, lda, batch, a_batch_stride, tn) != QMK_OK) return QMK_ERR_ARGS;
  a.C = C;
  a.ldc = ldc;
  a.c_batch = c_batch_stride;
  a.c_split = c_split_stride;
  a.n = n;
  a.rows = rows;
  a.kb_total = kb_total;
  a.kb_per_split = kbps;
  a.splits = splits;
  a.status = status;
  const int tiles_m = (n + kBM - 1) / kBM, tiles_n = (rows + tn - 1) / tn;
  const long long z = (long long)batch * splits;
  if (z > 65535) return qmk_internal_set_error(QMK_ERR_ARGS, "qmk_gemm: batch x splits too large");
  switch (tn) {
    case 32: return launch<32, 8>(a, tiles_m, tiles_n, (int)z, stream, dev);
    case 64: return launch<64, 8>(a, tiles_m, tiles_n, (int)z, stream, dev);
    case 128: return launch<128, 6>(a, tiles_m, tiles_n, (int)z, stream, dev);
    default: return launch<256, 4>(a, tiles_m, tiles_n, (int)z, stream, dev);
  }
}

extern "C" int qmk_gemm_bf16_nt(const void *W, long long ldw, long long w_batch_stride, int n, const void *A,
                                long long lda, long long a_batch_stride, int rows, int k, int batch, int splits,
                                float *C, long long ldc, long long c_batch_stride, long long c_split_stride,
                                unsigned *status, cudaStream_t stream) {
  qmk_internal_clear_error();
  const int rc = qmk_internal_gemm(W, ldw, w_batch_stride, n, A, lda, a_batch_stride, rows, k, batch, splits, C, ldc,
                                   c_batch_stride, c_split_stride, status, stream);
  return rc;
}
