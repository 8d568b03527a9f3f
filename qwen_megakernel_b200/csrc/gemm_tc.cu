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
// A tile is 128 x TN of C^T: W rows m0 .. m0+127 are the MMA's M = 128
// operand (TMEM lane = W row), A rows n0 .. n0+TN-1 the N operand (TMEM
// column = A row).  A persistent grid (one CTA per SM; three for prompt-sized
// GEMMs, see qmk_internal_gemm) walks the tiles; warp 0 (one lane) issues
// the TMA loads of 64-element K blocks, warp 1 the MMAs
// (4 of K = 16 per block) and tcgen05.commit, which frees a ring stage once
// its MMAs have read it and hands a finished accumulator to the epilogue
// warps 2-5, which read it (tcgen05.ld, lane = W row) and store C column by
// column, 32 consecutive W rows per warp store (coalesced).
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
constexpr int kWBytes = kBM * kBK * 2;   // 16 KB
constexpr unsigned long long kWaitNs = 1000000000ull;

struct Args {
  CUtensorMap tw;  // W: dims {K, n, batch}, box {64, 128, 1}
  CUtensorMap ta;  // A: dims {K, rows, batch}, box {64, TN, 1}
  float *C;
  long long ldc, c_batch, c_split;
  int n, rows, kb_total, kb_per_split, splits, batch;
  // causal prompt attention (A rows = query rows, row i at position i % causal_R):
  //   1: W rows = key positions; a tile whose keys all lie after every query
  //      of the tile is skipped (its scores are masked, C is left unwritten);
  //   2: K = key positions; a tile's K range stops after its last query's
  //      position (P is zero beyond it).
  int causal, causal_R;
  int w_static;  // W does not depend on the previous kernel (model weights): prefetch it before pdl_wait
  unsigned *status;
};

// Largest position (row % R) among A rows [n0, n1).
__device__ __forceinline__ int max_pos(int n0, int n1, int R) {
  return (n0 / R != (n1 - 1) / R) ? R - 1 : (n1 - 1) % R;
}

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
static_assert(2 * 8 * 8 + 5 * 8 + 8 <= 256, "barrier area");

// Persistent, warp-specialized: CTA c of G processes tiles c, c + G, ...
// (activation tile fastest, so the CTAs that share a weight tile run at the
// same time and read it from L2).  Warp 0: TMA producer (one lane); warp 1:
// MMA issuer; warps 2-5: epilogue (warp w reads TMEM lane quarter w % 4).
// Two TMEM accumulators: the epilogue of tile i overlaps the MMAs of tile
// i + 1.
constexpr int kPThreads = 192;

template <int TN, int STAGES>
__global__ void __launch_bounds__(kPThreads, 1) gemm_kernel(const __grid_constant__ Args g) {
  constexpr int kABytes = TN * kBK * 2;
  constexpr int kStageBytes = kWBytes + kABytes;
  constexpr int kAccCols = tmem_cols<TN>();
  constexpr int kCols = 2 * kAccCols;
  static_assert(TN % 32 == 0 && TN <= 256, "TN: 32 .. 256 in steps of 32");
  static_assert(kStageBytes % 1024 == 0, "stages must keep 1 KB swizzle-atom alignment");
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * kStageBytes);
  uint64_t *empty = full + STAGES;
  uint64_t *acc_full = empty + STAGES;  // [2] MMA -> epilogue (tcgen05.commit)
  uint64_t *acc_empty = acc_full + 2;   // [2] epilogue -> MMA (4 warps)
  uint64_t *drain = acc_empty + 2;      // MMA issuer: all its MMAs done
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tiles_m = (g.n + kBM - 1) / kBM, tiles_n = (g.rows + TN - 1) / TN;

  if (tid == 0) {
    for (int st = 0; st < STAGES; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(drain, 1);
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
  const int tiles_mn = tiles_m * tiles_n;
  const int ntiles = tiles_mn * g.splits * g.batch;
  auto decode_tile = [&](int t, int &tm, int &tn, int &bz, int &sp) {
    tn = t % tiles_n;
    int r = t / tiles_n;
    tm = r % tiles_m;
    r /= tiles_m;
    sp = r % g.splits;
    bz = r / g.splits;
  };
  // K blocks of tile t (split sp, activation tile tn); 0 = the tile is skipped
  auto kblocks = [&](int tm, int tn, int sp, int &kb0, int &nkb) {
    kb0 = sp * g.kb_per_split;
    int kb1 = min(g.kb_total, kb0 + g.kb_per_split);
    if (g.causal) {
      const int mp = max_pos(tn * TN, min(g.rows, (tn + 1) * TN), g.causal_R);
      if (g.causal == 1 && tm * kBM > mp) kb1 = kb0;
      if (g.causal == 2) kb1 = min(kb1, mp / kBK + 1);
    }
    nkb = max(0, kb1 - kb0);
  };

  pdl_trigger();
  if (warp == 0) {
    if (lane == 0) {
      // TMA producer: one continuous ring position over all tiles.  The
      // weight blocks of the first ring stages do not depend on the previous
      // kernel: they are requested before waiting for it (pdl_wait).
      uint32_t gk = 0;  // k blocks issued so far
      int pre = 0;      // stages of the first tile whose W block is already requested
      if (g.w_static && blockIdx.x < ntiles) {
        int tm, tn, bz, sp, kb0, nkb;
        decode_tile(blockIdx.x, tm, tn, bz, sp);
        kblocks(tm, tn, sp, kb0, nkb);
        pre = min(nkb, STAGES);
        for (int i = 0; i < pre; ++i) {
          mbar_arrive_expect_tx(&full[i], kStageBytes);
          tma_load_3d(smem + i * kStageBytes, &g.tw, (kb0 + i) * kBK, tm * kBM, bz, &full[i]);
        }
      }
      pdl_wait();
      for (int t = blockIdx.x; t < ntiles && !*abort_flag; t += gridDim.x) {
        int tm, tn, bz, sp, kb0, nkb;
        decode_tile(t, tm, tn, bz, sp);
        kblocks(tm, tn, sp, kb0, nkb);
        for (int i = 0; i < nkb; ++i, ++gk) {
          const int st = gk % STAGES;
          const uint32_t use = gk / STAGES;
          uint8_t *sw = smem + st * kStageBytes;
          if (gk < (uint32_t)pre) {  // W already requested: only the activation block
            tma_load_3d(sw + kWBytes, &g.ta, (kb0 + i) * kBK, tn * TN, bz, &full[st]);
            continue;
          }
          if (use > 0 && !wait_bar(&empty[st], (use - 1) & 1, abort_flag)) {
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[st], kStageBytes);
          tma_load_3d(sw, &g.tw, (kb0 + i) * kBK, tm * kBM, bz, &full[st]);
          tma_load_3d(sw + kWBytes, &g.ta, (kb0 + i) * kBK, tn * TN, bz, &full[st]);
        }
      }
      if (gk < (uint32_t)pre) gk = pre;  // (abort before the prefetched stages were completed)
      // copies in flight must land before the CTA's shared memory goes away
      for (uint32_t i = (gk > (uint32_t)STAGES ? gk - STAGES : 0u); i < gk; ++i) {
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&full[i % STAGES], (i / STAGES) & 1))
          if (global_timer_ns() - t0 > kWaitNs) break;
      }
    }
  } else if (warp == 1) {
    // MMA issuer: the converged warp issues, one elected lane executes
    pdl_wait();
    const uint32_t idesc = mma_idesc_bf16(kBM, TN);
    uint32_t gk = 0;
    int it = 0;  // tiles of this CTA
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
      int tm, tn, bz, sp, kb0, nkb;
      decode_tile(t, tm, tn, bz, sp);
      kblocks(tm, tn, sp, kb0, nkb);
      if (nkb == 0) continue;  // skipped tile: no accumulator
      const int b = it & 1;
      const uint32_t buse = (uint32_t)it >> 1;
      bool ok = true;
      if (lane == 0 && buse > 0) ok = wait_bar(&acc_empty[b], (buse - 1) & 1, abort_flag);
      if (!__shfl_sync(0xffffffffu, (int)ok, 0)) {
        if (lane == 0) *abort_flag = 1;
        break;
      }
      tc_fence_after_sync();
      const uint32_t d = tmem + (uint32_t)(b * kAccCols);
      for (int i = 0; i < nkb; ++i, ++gk) {
        const int st = gk % STAGES;
        ok = true;
        if (lane == 0) ok = wait_bar(&full[st], (gk / STAGES) & 1, abort_flag);
        if (!__shfl_sync(0xffffffffu, (int)ok, 0)) break;
        tc_fence_after_sync();
        const uint8_t *sw = smem + st * kStageBytes;
        const uint64_t ad = smem_desc_sw128(smem_addr(sw), 1024u);
        const uint64_t bd = smem_desc_sw128(smem_addr(sw + kWBytes), 1024u);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) tc_mma_bf16_warp(d, ad + 2u * kk, bd + 2u * kk, idesc, i > 0 || kk > 0);
        tc_commit_warp(&empty[st]);
      }
      tc_commit_warp(&acc_full[b]);
      ++it;
      if (!ok) {
        if (lane == 0) *abort_flag = 1;
        break;
      }
    }
    tc_commit_warp(drain);  // completes once every MMA issued above has
  } else {
    // epilogue warps 2..5: TMEM lane quarter q = warp % 4, W rows 32q .. 32q + 31
    pdl_wait();  // C may still be read by the previous kernel
    const int q = warp & 3;
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
      int tm, tn, bz, sp, kb0, nkb;
      decode_tile(t, tm, tn, bz, sp);
      kblocks(tm, tn, sp, kb0, nkb);
      if (nkb == 0) continue;
      const int b = it & 1;
      const uint32_t buse = (uint32_t)it >> 1;
      bool ok = true;
      if (lane == 0) ok = wait_bar(&acc_full[b], buse & 1, abort_flag);
      ok = __shfl_sync(0xffffffffu, (int)ok, 0) && *abort_flag == 0;
      if (!ok) break;
      tc_fence_after_sync();
      const int m = tm * kBM + 32 * q + lane;
      float *cb = g.C + (size_t)bz * (size_t)g.c_batch + (size_t)sp * (size_t)g.c_split;
      const int n0 = tn * TN;
#pragma unroll
      for (int c0 = 0; c0 < TN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * kAccCols + c0), r);
        if (m < g.n) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int col = n0 + c0 + j;
            if (col < g.rows) cb[(size_t)col * (size_t)g.ldc + m] = __uint_as_float(r[j]);
          }
        }
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
      ++it;
    }
  }
  // Every MMA the issuer started must finish before TMEM is freed (bounded).
  if (warp == 1 && lane == 0) {
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(drain, 0))
      if (global_timer_ns() - t0 > kWaitNs) break;
  }
  if (tid == 0 && *abort_flag && g.status) atomicOr(g.status, QMK_BATCH_TIMEOUT);
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

template <int TN, int STAGES, int CPS = 1>
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
  static int sms[kMaxDevices] = {};
  if (!sms[dev] && cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return qmk_internal_set_error(QMK_ERR_CUDA, "SM count");
  const long long total = (long long)tiles_m * tiles_n * z;
  const long long slots = (long long)CPS * sms[dev];  // CPS CTAs per SM (shared memory and TMEM permitting)
  const int grid = (int)(total < slots ? total : slots);
  // programmatic stream serialization: see the producer's weight prefetch
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kPThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, gemm_kernel<TN, STAGES>, a);
  if (e != cudaSuccess) return qmk_internal_set_error(QMK_ERR_CUDA, cudaGetErrorString(e));
  e = cudaGetLastError();
  if (e != cudaSuccess) return qmk_internal_set_error(QMK_ERR_CUDA, cudaGetErrorString(e));
  return QMK_OK;
}

}  // namespace qgemm

// Internal entry (batch.cu): see qmk_gemm_bf16_nt in include/qwen_megakernel.h.
__attribute__((visibility("hidden"))) int qmk_internal_gemm(
    const void *W, long long ldw, long long w_batch_stride, int n, const void *A, long long lda,
    long long a_batch_stride, int rows, int k, int batch, int splits, float *C, long long ldc, long long c_batch_stride,
    long long c_split_stride, unsigned *status, cudaStream_t stream, int causal, int causal_R, int w_static) {
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
  // Activation tile: the rows rounded up to 32 / 64 / 128.  More than 128
  // rows (prompts) use 64-row tiles with three CTAs per SM (3 ring stages
  // each; their producers and MMA issuers overlap each other's waits).
  // 1024-token prefill, measured: one CTA per SM with 256-row tiles 9.95 ms,
  // with 128-row tiles 8.9 ms; 128-row tiles x 2 CTAs x 3 stages 8.2 ms,
  // x 2 stages 11.0 ms; 64-row tiles x 4 CTAs x 2 stages 9.0 ms, x 2 CTAs x
  // 4 stages 7.9 ms, x 3 CTAs x 3 stages 7.7 ms.
  const bool big = rows > 128;
  const int tn = big ? 64 : rows <= 32 ? 32 : rows <= 64 ? 64 : 128;
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
  a.batch = batch;
  a.causal = (causal == 1 || causal == 2) && causal_R > 0 ? causal : 0;
  a.causal_R = causal_R;
  a.w_static = w_static ? 1 : 0;
  a.status = status;
  const int tiles_m = (n + kBM - 1) / kBM, tiles_n = (rows + tn - 1) / tn;
  const long long z = (long long)batch * splits;
  if ((long long)tiles_m * tiles_n * z > (1LL << 31) - 1)
    return qmk_internal_set_error(QMK_ERR_ARGS, "qmk_gemm: too many tiles");
  if (big) return launch<64, 3, 3>(a, tiles_m, tiles_n, (int)z, stream, dev);
  switch (tn) {
    case 32: return launch<32, 8>(a, tiles_m, tiles_n, (int)z, stream, dev);
    case 64: return launch<64, 8>(a, tiles_m, tiles_n, (int)z, stream, dev);
    default: return launch<128, 6>(a, tiles_m, tiles_n, (int)z, stream, dev);
  }
}

extern "C" int qmk_gemm_bf16_nt(const void *W, long long ldw, long long w_batch_stride, int n, const void *A,
                                long long lda, long long a_batch_stride, int rows, int k, int batch, int splits,
                                float *C, long long ldc, long long c_batch_stride, long long c_split_stride,
                                unsigned *status, cudaStream_t stream) {
  qmk_internal_clear_error();
  const int rc = qmk_internal_gemm(W, ldw, w_batch_stride, n, A, lda, a_batch_stride, rows, k, batch, splits, C, ldc,
                                   c_batch_stride, c_split_stride, status, stream, 0, 0, 0);
  return rc;
}
