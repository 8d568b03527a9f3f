// Persistent decode megakernel for Qwen3-0.6B on B200 (sm_100a), plus the C ABI.
//
// Structure (one cooperative launch runs `num_steps` greedy decode steps):
//   * one CTA per SM (148 on B200), 256 threads: 7 consumer warps + 1 producer warp;
//   * the producer warp streams every byte the CTA will read (its slice of each
//     weight matrix, its KV-cache chunk, its LM-head rows) through a 6 x 32 KB
//     shared-memory ring with 1-D TMA bulk copies (cp.async.bulk) and mbarriers.
//     Weights do not depend on activations, so the ring runs ahead across every
//     dependency point and keeps HBM busy while consumers wait;
//   * there is no grid barrier.  Each phase output element is written exactly
//     once per (step, layer) as an 8-byte word (fp32 value | epoch flag << 32);
//     consumers poll the words they need until the flag matches.  A dependency
//     therefore costs one L2 write->read latency instead of fence + atomic
//     barrier + re-read.
//   * per layer: P1 RMSNorm+QKV rows -> P2 QK-norm/RoPE/KV-append + split-KV
//     attention items -> P2.5 merge of the split partials -> P3 O-proj rows +
//     residual -> P4 RMSNorm + gate/up rows + SiLU -> P5 down rows + residual;
//     after the last layer the final RMSNorm + tied LM head + grid-wide argmax.
//   * the layer GEMVs run on the CUDA cores straight from the ring tiles (fp32
//     FMA over bf16 weights, input vector fp32 in shared memory); the LM head,
//     which streams 311 MB and is bound by HBM, runs on the tensor cores
//     (tcgen05.mma with TMEM accumulators);
//   * a second instance decodes 4 sequences per step (qmk_run_batch): every
//     weight tile is read once for all 4, q|k|v, gate/up and the LM head run
//     on the tensor cores with the sequences as the MMA's N columns, O and
//     down stay K-splits on the CUDA cores.
//
// Numerics follow the reference kernel (fp32 activations and accumulation,
// bf16 weights, bf16 K/V cache, bf16 cos/sin tables), except that the residual
// stream between layers stays fp32 (the reference rounds it to bf16,
// csrc/kernel.cu:859), which keeps the result closer to the fp32 evaluation of
// the HF PyTorch path the reference compares against.
//
// Every wait is bounded: an mbarrier or flag wait that exceeds timeout_ns
// records an error in the workspace control block, poisons the CTA (no further
// copies or stores), drains its in-flight copies and exits; the last CTA to
// exit publishes the error to the host-visible status block.

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "qmk_device.cuh"
#include "qmk_schedule.h"
#include "qwen_megakernel.h"

namespace qmk {

#ifndef QMK_CONSUMER_WARPS
#define QMK_CONSUMER_WARPS 7
#endif
constexpr int kConsumerWarps = QMK_CONSUMER_WARPS;  // + 1 producer warp
static_assert(kConsumerWarps >= 7 && kConsumerWarps <= 15, "the LM head needs 4 TMEM reader + 3 issuer warps");
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads + 32;

__device__ __forceinline__ void consumer_sync() { named_sync<kConsumerThreads>(); }
constexpr float kRmsEps = 1e-6f;
constexpr float kLog2e = 1.4426950408889634f;
constexpr unsigned long long kDefaultTimeoutNs = 1000000000ull;  // 1 s
constexpr unsigned kEpochWrap = 0xF0000000u;

enum Site : unsigned {
  kSiteFull = 1,
  kSiteEmpty = 2,
  kSiteX = 3,
  kSiteQKV = 4,
  kSitePart = 5,
  kSiteAtt = 6,
  kSiteA = 7,
  kSiteM = 8,
  kSiteArg = 9,
  kSiteKVReady = 10,
  kSiteToken = 11,
  kSiteMma = 12,
  kSiteTopk = 13,
};

struct Params {
  const __nv_bfloat16 *embed;
  const LDGLayerWeights *layers;
  const __nv_bfloat16 *final_norm;
  const __nv_bfloat16 *lm_head;
  const __nv_bfloat16 *cos_t;
  const __nv_bfloat16 *sin_t;
  __nv_bfloat16 *k_cache;
  __nv_bfloat16 *v_cache;
  uint8_t *ws;
  const int *forced;
  int n_forced;
  int first_token;
  int start_pos;
  int num_steps;
  int num_layers;
  int max_seq_len;
  float attn_scale;
  int splits;
  int *out_log;
  int *out_token;
  float *logits;
  float *final_hidden;
  QmkStatus *status;
  unsigned long long timeout_ns;
  int debug_stall;
  unsigned long long *trace;  // optional [ncta][kTraceStride] globaltimer stamps
  int trace_step;
  unsigned poll_backoff_ns;
  unsigned tuning;
  float inv_temp;       // sampling: 1 / temperature, 0 = greedy
  unsigned long long seed;
  int top_k;            // sampling restricted to the top_k logits (0: all)
  int eos_token;        // stop after a generated token equal to this (-1: never)
  int *steps_done;      // optional: steps executed (< num_steps after an EOS stop)
  // Batched instance (NB > 1 sequences): per-sequence start positions, the
  // elements between sequences' caches and the step-0 tokens (device [NB]).
  int start_pos_b[kMaxSeqs];
  long long cache_seq_stride;
  const int *first_tokens_b;
};

// Dynamic shared memory plan (bytes).
constexpr int kSmRing = 0;
constexpr int kSmX = kNumSlots * kSlotBytes;   // layer input residual, fp32 [1024]
constexpr int kSmA = kSmX + 4 * kHidden;       // post-attention residual, fp32 [1024]
constexpr int kSmAtt = kSmA + 4 * kHidden;     // attention output, fp32 [2048]
constexpr int kSmU = kSmAtt + 4 * kQSize;      // MLP intermediate / attention scratch, fp32 [3072]
constexpr int kSmXW = kSmU + 4 * kInter;       // RMSNorm input times the norm weights, fp32 [1024]
constexpr int kSmMisc = kSmXW + 4 * kHidden;
// misc (bytes): full/empty mbarriers, per-warp argmax (value, index), block
// reductions (4 call sites), tensor-core completion / TMEM-free mbarriers,
// TMEM base address, K-split partial row sums.
constexpr int kMiscBestV = 16 * kNumSlots;
constexpr int kMiscBestI = kMiscBestV + 64;
constexpr int kMiscRed = kMiscBestI + 64;  // [4][16] fp32
constexpr int kMiscMmaBar = kMiscRed + 256;  // [kTmemBufs] tensor-core completion (count 1)
constexpr int kMiscTmemFree = kMiscMmaBar + 64; // [kTmemBufs] accumulator read by warps 0-3 (count 4)
constexpr int kMiscTmem = kMiscTmemFree + 64;
static_assert(kConsumerWarps <= 16, "per-warp misc slots hold 16 warps");
constexpr int kMiscPart = kMiscTmem + 64;  // [2][16][kKsplitGroupRows] fp32: per-warp partial row sums (K split)
constexpr int kKsplitRows = 4;       // rows of a K-split GEMV register batch
constexpr int kKsplitGroupRows = 8;  // rows whose partial sums meet behind one barrier
constexpr int kMiscRes = kMiscPart + 2 * 16 * kKsplitGroupRows * 4;  // [2][kMaxSeqs][16] fp32: residual rows (batched)
constexpr int kMaxResRows = 8;   // O / down rows per CTA the batched instance keeps residuals of (>= 128 CTAs)
constexpr int kMiscBytes = kMiscRes + 2 * kMaxSeqs * kMaxResRows * 4;
// A CUDA-core GEMV phase holds all of its ring tiles at once: they must fit
// in the ring for the smallest grid.
static_assert((kQKVRows / kMinCtas + 1 + kQKVTileRows - 1) / kQKVTileRows <= kNumSlots, "q|k|v tiles exceed the ring");
static_assert((kHidden / kMinCtas + 1 + kOTileRows - 1) / kOTileRows <= kNumSlots, "O tiles exceed the ring");
static_assert((kInter / kMinCtas + kGUTileRows - 1) / kGUTileRows <= kNumSlots, "gate/up tiles exceed the ring");
static_assert((kHidden / kMinCtas + 1 + kDTileRows - 1) / kDTileRows <= kNumSlots, "down tiles exceed the ring");
#ifndef QMK_LM_PREFETCH_TILES
#define QMK_LM_PREFETCH_TILES 16
#endif
constexpr int kLmPrefetchTiles = QMK_LM_PREFETCH_TILES;  // LM-head tiles per CTA prefetched into L2
constexpr int kLmPrefetchLayers = 4;                     // ... spread over the last layers
constexpr int kTmemBufs = 8;       // GEMV units (M blocks) in flight
constexpr int kTmemBufCols = 64;   // D of one unit: 128 lanes x N (<= 48) fp32 columns
constexpr int kTmemCols = kTmemBufs * kTmemBufCols;
constexpr int kSmBytes = kSmMisc + kMiscBytes;
// 227 KB per block on sm_100, of which the kernel's static __shared__ data
// (argmax exchange, abort/stop flags) takes up to 1 KB.
static_assert(kSmBytes + 1024 <= 232448, "shared memory plan exceeds the sm_100 per-block limit");

// Attention scratch inside the U region (floats).
constexpr int kUQ = 0;      // q, 2 heads [256]
constexpr int kUK = 256;    // k [128]
constexpr int kUV = 384;    // v [128]
constexpr int kUKn = 512;   // new k after norm/RoPE, one bf16 cache row (256 B)
constexpr int kUVn = 640;   // new v, one bf16 cache row (256 B)
constexpr int kUPW = 768;   // per-warp partials [8][260]
// (the per-warp partials may run on into the x*w buffer, free during attention)
static_assert(kUPW + kConsumerWarps * kPartWords <= kInter + kHidden, "attention scratch too large");
static_assert(kMaxSplits * kMergeWordsPerSplit <= kInter, "merge scratch too large");

// Optional timeline trace (one step): per CTA, per layer 16 slots
//   0 P1 input ready   1 P1 done   2 P2 q/k/v ready  3 P2 done
//   4 P2.5 ready       5 P2.5 done 6 P3 ATT ready    7 P3 done
//   8 P4 A ready       9 P4 done  10 P5 M ready     11 P5 done
//  12 producer: first tile of the layer issued  13 producer: last tile issued
// and after the last layer (slot base num_layers*16): 0 LM input ready,
// 1 LM done, 3 producer LM first tile, 4 producer LM last tile, 5 step start.
// Then, per ring tile k of the step (k < kTraceTiles): [kTraceTileBase + 2k]
// consumer warp 0 starts waiting for it, [+2k+1] it has landed,
// [kTraceTileBase + 2*kTraceTiles + k] the producer issued its copy and
// [kTraceTileBase + 3*kTraceTiles + k] consumer warp 0 released it; for
// tensor-core tiles [+4*kTraceTiles + k] thread 0 read its accumulator and
// [+5*kTraceTiles + k] finished its rows.
constexpr int kTraceTiles = 512;
constexpr int kTraceTileBase = (kMaxLayers + 1) * 16;
constexpr int kTraceStride = kTraceTileBase + 6 * kTraceTiles;

struct Ctx {
  uint8_t *ring;
  uint64_t *full;
  uint64_t *empty;
  volatile int *abort_flag;
  volatile int *stop_step;  // first step not to run (EOS seen), INT_MAX = none
  float *warp_best_v;
  int *warp_best_i;
  int *token_slot;
  Ctrl *ctrl;
  uint64_t *wX, *wQKV, *wPart, *wAtt, *wA, *wM, *wArg;
  uint64_t *wTopk;  // top-k sampling: [cta][top_k] candidate keys
  int cta, ncta;
  unsigned E0;
  unsigned long long timeout_ns;
  int cur_layer;
  unsigned long long *trace;  // this CTA's trace row, or nullptr
  uint32_t trace_tile0;       // ring tile index at the start of the traced step
  unsigned poll_backoff_ns;   // sleep between failed dataflow polls (0: spin)
  unsigned tuning;            // QmkRunArgs.tuning
  uint64_t *mma_bar;          // [kTmemBufs] tensor-core completion (tcgen05.commit)
  uint64_t *tmem_free;        // [kTmemBufs] accumulator buffer read out
  uint32_t tmem;              // TMEM base address of the GEMV accumulators
};

__device__ __forceinline__ unsigned epoch_of(const Ctx &c, int step, int layer, int num_layers) {
  return c.E0 + 1u + (unsigned)step * (unsigned)(num_layers + 1) + (unsigned)layer;
}

// Hardware approximations (ex2.approx / rcp.approx, ~2 ulp) for the softmax
// and SiLU: they sit on dependent chains where libm's accurate sequences
// cost several times the latency.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float fast_rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Standard Gumbel noise of vocabulary row `idx` at cache position `pos` for
// sampling seed `seed`: u from the splitmix64 finalizer (Steele, Lea and
// Flood 2014) of a (seed, position, index) key, 24 bits in (0, 1), then
// -log(-log(u)).  argmax_i(logit_i / T + g_i) is an exact draw from
// softmax(logits / T) (the Gumbel-max trick), so sampling reuses the greedy
// argmax exchange unchanged; the key depends on the position, not on the
// launch, so a sequence samples the same tokens however it is split into
// launches.
__device__ __forceinline__ float gumbel_noise(unsigned long long seed, int pos, int idx) {
  unsigned long long z = seed ^ (((unsigned long long)(unsigned)pos << 20) | (unsigned)idx);
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  const float u = ((float)(unsigned)(z >> 40) + 0.5f) * (1.0f / 16777216.0f);
  return -logf(-logf(u));
}

__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned *p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// QmkRunArgs.tuning bit 4: trace stamps in SM clock cycles (%clock64) instead
// of %globaltimer ns.  The global timer ticks in 256 ns steps on B200, too
// coarse for the sub-microsecond intervals inside a phase; clock64 resolves
// them but is per SM, so only differences within one CTA are meaningful.
constexpr unsigned kTuneTraceClock = 16u;

__device__ __forceinline__ uint64_t trace_now(const Ctx &c) {
  if (c.tuning & kTuneTraceClock) {
    uint64_t t;
    asm volatile("mov.u64 %0, %%clock64;" : "=l"(t));
    return t;
  }
  return global_timer_ns();
}

__device__ __forceinline__ void trace_stamp(const Ctx &c, bool active, int slot) {
  if (active && c.trace) c.trace[slot] = trace_now(c);
}

// Slow paths stay out of line: the kernel cycles through all of its phases
// every layer, so code that is rarely executed should not sit in the hot
// instruction stream.
__device__ __noinline__ void raise_error_at(volatile int *abort_flag, Ctrl *ctrl, unsigned code,
                                            unsigned site, int cta, int layer) {
  *abort_flag = 1;
  if (atomicCAS(&ctrl->err_code, 0u, code) == 0u) {
    atomicExch(&ctrl->err_info, ((unsigned)cta << 16) | ((site & 0xffu) << 8) | ((unsigned)layer & 0xffu));
  }
}

__device__ __forceinline__ void raise_error(Ctx &c, unsigned code, unsigned site) {
  raise_error_at(c.abort_flag, c.ctrl, code, site, c.cta, c.cur_layer);
}

// Every 16th failed poll: abort / deadline / foreign-error checks (no sleep:
// a waiting warp only spins on its own poll, and a sleep would delay the
// wake-up).  Returns
// the (possibly newly set) deadline, or 0 when the wait must give up.
__device__ __noinline__ uint64_t wait_checkpoint(volatile int *abort_flag, Ctrl *ctrl, uint64_t deadline,
                                                 unsigned it, unsigned long long timeout_ns, unsigned site,
                                                 int cta, int layer) {
  if (*abort_flag) return 0;
  const uint64_t now = global_timer_ns();
  if (deadline == 0) {
    deadline = now + timeout_ns;
  } else if (now > deadline || it > (1u << 30)) {
    raise_error_at(abort_flag, ctrl, QMK_ERR_TIMEOUT, site, cta, layer);
    return 0;
  }
  if ((it & 1023u) == 0u && ld_relaxed_u32(&ctrl->err_code) != 0u) {
    *abort_flag = 1;  // another CTA failed: stop waiting for it
    return 0;
  }
  return deadline;
}

// Bounded-wait bookkeeping: call keep_going() once per failed poll.
struct Waiter {
  uint64_t deadline = 0;
  unsigned it = 0;
  __device__ __forceinline__ bool keep_going(Ctx &c, unsigned site) {
    ++it;
    if ((it & 15u) != 0u) return true;
    deadline = wait_checkpoint(c.abort_flag, c.ctrl, deadline, it, c.timeout_ns, site, c.cta, c.cur_layer);
    return deadline != 0;
  }
};

// ------------------------------------------------------------- ring (consumer)
// No abort pre-check here or in the other waits: a strong shared-memory
// access costs 80-170 SM cycles inside this kernel (measured), and the wait
// loops see an abort at their next checkpoint anyway.
__device__ __forceinline__ bool wait_full(Ctx &c, uint32_t tile) {
  bool ok = true;
  const uint32_t k = tile - c.trace_tile0;
  const bool stamp = c.trace && threadIdx.x == 0 && k < (uint32_t)kTraceTiles;
  if (stamp) c.trace[kTraceTileBase + 2 * k] = trace_now(c);
  const int slot = tile % kNumSlots;
  const unsigned par = (tile / kNumSlots) & 1u;
  Waiter w;
  while (!mbar_try_wait(&c.full[slot], par)) {
    if (!w.keep_going(c, kSiteFull)) {
      ok = false;
      break;
    }
  }
  if (stamp) c.trace[kTraceTileBase + 2 * k + 1] = trace_now(c);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void release_tile(Ctx &c, uint32_t tile, bool ok) {
  const uint32_t k = tile - c.trace_tile0;
  if (c.trace && threadIdx.x == 0 && k < (uint32_t)kTraceTiles)
    c.trace[kTraceTileBase + 3 * kTraceTiles + k] = trace_now(c);
  __syncwarp();
  if (ok && (threadIdx.x & 31) == 0) mbar_arrive(&c.empty[tile % kNumSlots]);
}

// wait_full for one thread (the tensor-core issuer).
__device__ __forceinline__ bool wait_full_one(Ctx &c, uint32_t tile) {
  if (*c.abort_flag) return false;
  const uint32_t k = tile - c.trace_tile0;
  const bool stamp = c.trace && k < (uint32_t)kTraceTiles;
  if (stamp) c.trace[kTraceTileBase + 2 * k] = trace_now(c);
  const int slot = tile % kNumSlots;
  const unsigned par = (tile / kNumSlots) & 1u;
  Waiter w;
  while (!mbar_try_wait(&c.full[slot], par)) {
    if (!w.keep_going(c, kSiteFull)) return false;
  }
  if (stamp) c.trace[kTraceTileBase + 2 * k + 1] = trace_now(c);
  return true;
}

__device__ __forceinline__ const uint8_t *slot_ptr(const Ctx &c, uint32_t tile) {
  return c.ring + (tile % kNumSlots) * kSlotBytes;
}

// ------------------------------------------------------------- GEMV (tcgen05)
// LM head: y = W x for the rows of one 32 KB ring tile runs on the 5th-generation
// tensor cores: tcgen05.mma (M = 128, N = 16S, K = 16, bf16 in, fp32
// accumulate in TMEM) with the tile's weights as the A operand exactly as
// the 1-D bulk copies deliver them and the activation vector as the B
// operand, both read through the 128-byte-swizzle descriptor:
//
//  * the tile is 16 "segments" of 2 KB (1024 weights): a row for K = 1024,
//    half a row for K = 2048, and for K = 3072 (rows at an 8 KB pitch) a
//    third of a row or an unused quarter.  Segment j, half h' (0/1) is the
//    1 KB swizzle atom at byte 2048j + 1024h': 8 lines of 128 bytes, line q
//    holding weights 512h' + 64q + (0..63) of the segment;
//  * M block h' of the tile = atoms (j, h') for j = 0..15 (SBO 2048 bytes):
//    MMA row 8j + q is line q of segment j, and 4 instructions walk K = 64;
//  * the descriptor's swizzle reads logical 16-byte chunk c of line q from
//    chunk c ^ q.  B line (s, g, q) holds part g (0 = hi, 1 = lo) of the 64
//    activations that line q of a segment in slot s multiplies, in plain
//    order, so its chunks are permuted the same way and
//    D[8j + q][16s + 8g + q] (s = slot of segment j) is the line's partial
//    dot product (the "diagonal" entries; the others are unused).  Slots:
//    one for K = 1024, the half for K = 2048, the third for K = 3072, so
//    N = 16, 32, 48;
//  * the fp32 activation x is split as x = hi + lo (two bf16 parts, the
//    second holding the rounding remainder of the first): products are exact
//    and the representation error of x is ~2^-17 relative.
// Both M blocks map TMEM lane 8j + q to segment j, so a row's dot product is
// the sum of the two blocks' diagonal entries over 8 lanes (one segment),
// 16 lanes (K = 2048) or a whole warp (K = 3072), added with shuffles.
//
// B operand ("bop") for K = 1024S: the lines of block h' are contiguous
// (1 KB groups of 8 lines, group 2S*h' + 2s + g), so element e (slice
// h = e >> 9 = 2s + h', line q = (e >> 6) & 7) has its hi part at
// bop_offset<S>(e) and its lo part 1024 bytes further; 4S KB in all.
enum TcKind : int { kTcRow = 0, kTcGU = 1, kTcHalf = 2, kTcQuarter = 3 };
enum TcOut : int { kOutQKV = 0, kOutO = 1, kOutGU = 2, kOutDown = 3, kOutLM = 4 };

template <int S>
__device__ __forceinline__ int bop_offset(int e) {
  const int h = e >> 9;
  return 1024 * (2 * S * (h & 1) + 2 * (h >> 1)) + 128 * ((e >> 6) & 7) + 2 * (e & 63);
}

__device__ __forceinline__ uint32_t bf2_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t *>(&v); }

// Split (v0, v1) into bf16 pairs hi and lo with v ~= hi + lo.
__device__ __forceinline__ void split_pair(float v0, float v1, uint32_t &hi, uint32_t &lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(v0, v1);
  const float2 hf = __bfloat1622float2(h);
  hi = bf2_bits(h);
  lo = bf2_bits(__floats2bfloat162_rn(v0 - hf.x, v1 - hf.y));
}

// Elements e, e+1 (e even) of the activation vector (K = 1024S) into the B
// operand.
template <int S>
__device__ __forceinline__ void store_bop_pair(uint8_t *bop, int e, float v0, float v1) {
  uint32_t hi, lo;
  split_pair(v0, v1, hi, lo);
  uint8_t *q = bop + bop_offset<S>(e);
  *reinterpret_cast<uint32_t *>(q) = hi;
  *reinterpret_cast<uint32_t *>(q + 1024) = lo;
}

// r[q] for a per-lane q in [0, 8), as a tree of selects (no local memory).
__device__ __forceinline__ float sel8(const uint32_t *r, int q) {
  const uint32_t a0 = (q & 1) ? r[1] : r[0], a1 = (q & 1) ? r[3] : r[2];
  const uint32_t a2 = (q & 1) ? r[5] : r[4], a3 = (q & 1) ? r[7] : r[6];
  const uint32_t b0 = (q & 2) ? a1 : a0, b1 = (q & 2) ? a3 : a2;
  return __uint_as_float((q & 4) ? b1 : b0);
}

// This lane's diagonal entry pair (hi + lo) of a GEMV accumulator with S
// slots at TMEM address taddr: columns 16*slot + q and 16*slot + 8 + q.
// All columns a warp needs are loaded with one wait.
template <int S>
__device__ __forceinline__ float tc_read(uint32_t taddr, int slot, int q) {
  if (S == 1) {
    uint32_t r[16];
    tmem_ld16(taddr, r);
    return sel8(r, q) + sel8(r + 8, q);
  } else {
    uint32_t r[32];
    tmem_ld32(taddr, r);
    float v = (slot == 0) ? sel8(r, q) + sel8(r + 8, q) : sel8(r + 16, q) + sel8(r + 24, q);
    if (S == 3) {
      uint32_t r2[16];
      tmem_ld16(taddr + 32u, r2);
      if (slot == 2) v = sel8(r2, q) + sel8(r2 + 8, q);
    }
    return v;
  }
}

// ------------------------------------------------------------- LL staging
enum StageMode : int {
  kStageSumSq = 1,     // fp32 copy into dst, returns sum of squares of the vector
  kStageFrag = 2,      // tensor-core B operand of the vector into bop
  kStageNormFrag = 3,  // fp32 copy into dst, B operand of x * w (norm weights
                       // prefetched in nw), returns sum of squares
  kStageNorm = 4,      // fp32 copy into dst, fp32 x * w into dst2 (passed as
                       // bop), returns sum of squares
  kStageCopy = 5,      // fp32 copy into dst
};

// All consumer threads: poll the N words of `src` until their flag equals
// `flag` (two words per 16-byte load) and store them per MODE, then
// consumer_sync().  The sum of squares is folded into that barrier (block
// reduction through red[kConsumerWarps], one array per call site) and taken
// in a fixed order whatever the order in which the words arrive.  B operand
// writes (K = N) are fenced for the async proxy before the barrier.
// Thread tid handles word pairs q = tid + k * kConsumerThreads.
// Norm-weight pairs of the words a thread stages (kStageNormFrag), by value.
struct NormPairs {
  uint32_t w[4];
};

template <int N, int MODE>
__device__ __forceinline__ float stage_vec(Ctx &c, float *dst, uint8_t *bop, const uint64_t *src, unsigned flag,
                                        unsigned site, float *red, NormPairs nw) {
  constexpr int kPairs = N / 2;
  constexpr int P = (kPairs + kConsumerThreads - 1) / kConsumerThreads;
  constexpr bool kSum = (MODE == kStageSumSq || MODE == kStageNormFrag || MODE == kStageNorm);
  static_assert(N % 2 == 0 && P <= 32, "stage_vec size");
  static_assert((MODE != kStageNormFrag && MODE != kStageNorm) || P <= 4, "norm-weight pairs per thread");
  const int tid = threadIdx.x;
  unsigned pending = 0;
#pragma unroll
  for (int k = 0; k < P; ++k)
    if (k * kConsumerThreads + tid < kPairs) pending |= 1u << k;
  float keep[kSum ? P : 1][2];
#pragma unroll
  for (int k = 0; k < (kSum ? P : 1); ++k) keep[k][0] = keep[k][1] = 0.f;
  uint64_t a0[P], b0[P];
  auto issue = [&](uint64_t (&a)[P], uint64_t (&b)[P]) {
#pragma unroll
    for (int k = 0; k < P; ++k) {
      a[k] = 0;
      b[k] = 0;
      if (pending & (1u << k)) ll_load2(src + 2 * (k * kConsumerThreads + tid), a[k], b[k]);
    }
  };
  auto check = [&](const uint64_t (&a)[P], const uint64_t (&b)[P]) {
#pragma unroll
    for (int k = 0; k < P; ++k) {
      if ((pending & (1u << k)) && ll_flag(a[k]) == flag && ll_flag(b[k]) == flag) {
        const int q = k * kConsumerThreads + tid;
        const float v0 = ll_value(a[k]), v1 = ll_value(b[k]);
        if (MODE != kStageFrag) reinterpret_cast<float2 *>(dst)[q] = make_float2(v0, v1);
        if (MODE == kStageFrag) store_bop_pair<N / 1024>(bop, 2 * q, v0, v1);
        if (MODE == kStageNormFrag) {
          const uint32_t wk = nw.w[k < 4 ? k : 3];
          store_bop_pair<N / 1024>(bop, 2 * q, v0 * bf_lo(wk), v1 * bf_hi(wk));
        }
        if (MODE == kStageNorm) {
          const uint32_t wk = nw.w[k < 4 ? k : 3];
          reinterpret_cast<float2 *>(bop)[q] = make_float2(v0 * bf_lo(wk), v1 * bf_hi(wk));
        }
        if (kSum) {
          keep[kSum ? k : 0][0] = v0;
          keep[kSum ? k : 0][1] = v1;
        }
        pending &= ~(1u << k);
      }
    }
  };
  Waiter w;
  while (pending) {
    issue(a0, b0);
    check(a0, b0);
    if (!pending) break;
    if (!w.keep_going(c, site)) break;
    if (c.poll_backoff_ns) __nanosleep(c.poll_backoff_ns);
  }
  if (MODE == kStageFrag || MODE == kStageNormFrag) fence_proxy_async_smem();
  if (kSum) {
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < (kSum ? P : 1); ++k) ss = fmaf(keep[k][0], keep[k][0], fmaf(keep[k][1], keep[k][1], ss));
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
  }
  consumer_sync();
  float total = 0.f;
  if (kSum) {
#pragma unroll
    for (int q = 0; q < kConsumerWarps; ++q) total += red[q];
  }
  return total;
}

// NV vectors of N words in one staging (batched instance): vector b's words
// at src + b * src_stride are polled together (pair q of the NV * N / 2 pairs
// by thread q % kConsumerThreads) and stored as fp32 at dst + b * N; with
// kStageNorm also x * w (w: the bf16 norm weight in global memory, fetched
// before the wait) at dst2 + b * N, with kStageNormFrag x * w as the
// tensor-core B operand of the NV vectors side by side (N = 1024, slot b =
// vector b: element e of vector b is element 1024 b + e of a K = 1024 NV
// operand, N = 16 NV columns) at dst2, fenced for the async proxy; and
// ss[b] = the sum of squares of vector b (per thread in pair order, per warp
// by butterfly, over the warps in warp order through red[b * 16 + warp]).
// One consumer barrier for all vectors.
template <int N, int NV, int MODE>
__device__ __forceinline__ void stage_vecs(Ctx &c, float *dst, float *dst2, const uint64_t *src, size_t src_stride,
                                           unsigned flag, unsigned site, float *red, const __nv_bfloat16 *nw,
                                           float (&ss)[NV]) {
  constexpr int kHalf = N / 2;  // pairs per vector
  constexpr int kPairs = NV * kHalf;
  constexpr int P = (kPairs + kConsumerThreads - 1) / kConsumerThreads;
  constexpr bool kFrag = (MODE == kStageNormFrag);
  constexpr bool kNorm = (MODE == kStageNorm || kFrag);
  static_assert((MODE == kStageNorm || MODE == kStageNormFrag || MODE == kStageCopy) && P <= 32 && NV <= 4,
                "stage_vecs");
  static_assert(!kFrag || N == 1024, "B operand of K = 1024 inputs");
  const int tid = threadIdx.x;
  unsigned pending = 0;
  uint32_t wn[kNorm ? P : 1];
#pragma unroll
  for (int k = 0; k < P; ++k) {
    const int q = k * kConsumerThreads + tid;
    if (q < kPairs) pending |= 1u << k;
    if (kNorm) wn[kNorm ? k : 0] = (q < kPairs) ? __ldg(reinterpret_cast<const unsigned *>(nw) + q % kHalf) : 0u;
  }
  float acc[NV];
#pragma unroll
  for (int b = 0; b < NV; ++b) acc[b] = 0.f;
  float keep[kNorm ? P : 1][2];
#pragma unroll
  for (int k = 0; k < (kNorm ? P : 1); ++k) keep[k][0] = keep[k][1] = 0.f;
  uint64_t a0[P], b0[P];
  auto addr = [&](int q) { return src + (size_t)(q / kHalf) * src_stride + 2 * (q % kHalf); };
  Waiter w;
  while (pending) {
#pragma unroll
    for (int k = 0; k < P; ++k) {
      a0[k] = 0;
      b0[k] = 0;
      if (pending & (1u << k)) ll_load2(addr(k * kConsumerThreads + tid), a0[k], b0[k]);
    }
#pragma unroll
    for (int k = 0; k < P; ++k) {
      if ((pending & (1u << k)) && ll_flag(a0[k]) == flag && ll_flag(b0[k]) == flag) {
        const int q = k * kConsumerThreads + tid;
        const int bq = q / kHalf, qq = q % kHalf;
        const float v0 = ll_value(a0[k]), v1 = ll_value(b0[k]);
        reinterpret_cast<float2 *>(dst + bq * N)[qq] = make_float2(v0, v1);
        if (kNorm) {
          const uint32_t wk = wn[kNorm ? k : 0];
          if (kFrag)
            store_bop_pair<NV>(reinterpret_cast<uint8_t *>(dst2), 2 * q, v0 * bf_lo(wk), v1 * bf_hi(wk));
          else
            reinterpret_cast<float2 *>(dst2 + bq * N)[qq] = make_float2(v0 * bf_lo(wk), v1 * bf_hi(wk));
          keep[kNorm ? k : 0][0] = v0;
          keep[kNorm ? k : 0][1] = v1;
        }
        pending &= ~(1u << k);
      }
    }
    if (!pending) break;
    if (!w.keep_going(c, site)) break;
  }
  if (kFrag) fence_proxy_async_smem();
  if (kNorm) {
#pragma unroll
    for (int k = 0; k < P; ++k) {
      const int bq = (k * kConsumerThreads + tid) / kHalf;  // >= NV for pairs past the end (keep = 0)
      const float s2 = fmaf(keep[kNorm ? k : 0][0], keep[kNorm ? k : 0][0], keep[kNorm ? k : 0][1] * keep[kNorm ? k : 0][1]);
#pragma unroll
      for (int b = 0; b < NV; ++b) acc[b] += (bq == b) ? s2 : 0.f;
    }
#pragma unroll
    for (int b = 0; b < NV; ++b) {
      const float t = warp_sum(acc[b]);
      if ((tid & 31) == 0) red[b * 16 + (tid >> 5)] = t;
    }
  }
  consumer_sync();
#pragma unroll
  for (int b = 0; b < NV; ++b) {
    float total = 0.f;
    if (kNorm) {
#pragma unroll
      for (int q = 0; q < kConsumerWarps; ++q) total += red[b * 16 + q];
    }
    ss[b] = total;
  }
}

// Norm weights (bf16 pairs) of the word pairs thread `tid` stages
// (q = tid + j * kConsumerThreads), fetched before the dataflow wait.
__device__ __forceinline__ NormPairs load_norm_pairs(const __nv_bfloat16 *nw, int tid) {
  NormPairs r;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int q = tid + j * kConsumerThreads;
    r.w[j] = (q < kHidden / 2) ? __ldg(reinterpret_cast<const unsigned *>(nw) + q) : 0u;
  }
  return r;
}

// Slot `slot` of a B operand with S inputs side by side (K = 1024 S) <- x * w
// (K = 1024); the caller fences it for the tensor cores and publishes it
// with its next consumer_sync.
template <int S>
__device__ __forceinline__ void build_norm_bop_slot(uint8_t *bop, int slot, const float *x, const NormPairs &nw,
                                                    int tid) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int q = tid + j * kConsumerThreads;
    if (q < kHidden / 2) {
      const float2 v = reinterpret_cast<const float2 *>(x)[q];
      store_bop_pair<S>(bop, 1024 * slot + 2 * q, v.x * bf_lo(nw.w[j]), v.y * bf_hi(nw.w[j]));
    }
  }
}

// xw <- x * w (the RMSNorm weight; 1/rms is applied to the GEMV results),
// fp32; the caller's next consumer_sync publishes it.  K = 1024.
__device__ __forceinline__ void build_norm_xw(float *xw, const float *x, const NormPairs &nw, int tid) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int q = tid + j * kConsumerThreads;
    if (q < kHidden / 2) {
      const float2 v = reinterpret_cast<const float2 *>(x)[q];
      reinterpret_cast<float2 *>(xw)[q] = make_float2(v.x * bf_lo(nw.w[j]), v.y * bf_hi(nw.w[j]));
    }
  }
}

// Warp sums of four per-lane values v[0..3] (rows of a batch): lane l
// returns the sum over all lanes of v[2 ((l >> 4) & 1) + ((l >> 3) & 1)].
// Each level adds the same pairs in the same order on every run.
__device__ __forceinline__ float reduce4_transpose(const float (&v)[4]) {
  const int lane = threadIdx.x & 31;
  const bool hi16 = (lane & 16) != 0, hi8 = (lane & 8) != 0;
  float w[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const float send = hi16 ? v[j] : v[j + 2];
    const float keep = hi16 ? v[j + 2] : v[j];
    w[j] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
  const float send = hi8 ? w[0] : w[1];
  float u = (hi8 ? w[1] : w[0]) + __shfl_xor_sync(0xffffffffu, send, 8);
  u += __shfl_xor_sync(0xffffffffu, u, 4);
  u += __shfl_xor_sync(0xffffffffu, u, 2);
  u += __shfl_xor_sync(0xffffffffu, u, 1);
  return u;
}

// Sums over the 8 lanes of an aligned lane group of four per-lane values
// v[0..3]: lane q (= lane & 7) of the group returns the group's sum of
// v[q >> 1].  Three levels of one exchange each (4 shuffles), the same
// pairs added in the same order on every run.
__device__ __forceinline__ float reduce4_oct(const float (&v)[4]) {
  const int q = threadIdx.x & 7;
  const bool h4 = (q & 4) != 0, h2 = (q & 2) != 0;
  const float a0 = (h4 ? v[2] : v[0]) + __shfl_xor_sync(0xffffffffu, h4 ? v[0] : v[2], 4);
  const float a1 = (h4 ? v[3] : v[1]) + __shfl_xor_sync(0xffffffffu, h4 ? v[1] : v[3], 4);
  float u = (h2 ? a1 : a0) + __shfl_xor_sync(0xffffffffu, h2 ? a0 : a1, 2);
  u += __shfl_xor_sync(0xffffffffu, u, 1);
  return u;
}

// s0/s1 += 4 bf16 weights (w, two pairs) times 4 fp32 inputs (x), even and
// odd elements in separate chains.
__device__ __forceinline__ void dot4(float &s0, float &s1, const uint2 w, const float4 x) {
  s0 = fmaf(x.x, bf_lo(w.x), s0);
  s1 = fmaf(x.y, bf_hi(w.x), s1);
  s0 = fmaf(x.z, bf_lo(w.y), s0);
  s1 = fmaf(x.w, bf_hi(w.y), s1);
}

// Poll up to K words per thread at arbitrary addresses: word i (i < n) of the
// list is fetched by consumer thread i % kConsumerThreads from addr(i) and
// stored to dst[i].
template <int K, typename AddrFn>
__device__ void stage_list(Ctx &c, float *dst, int n, AddrFn addr, unsigned flag, unsigned site) {
  const int tid = threadIdx.x;
  unsigned pending = 0;
#pragma unroll
  for (int k = 0; k < K; ++k)
    if (k * kConsumerThreads + tid < n) pending |= 1u << k;
  uint64_t v0[K];
  auto issue = [&](uint64_t (&v)[K]) {
#pragma unroll
    for (int k = 0; k < K; ++k) {
      v[k] = 0;
      if (pending & (1u << k)) v[k] = ll_load(addr(k * kConsumerThreads + tid));
    }
  };
  auto check = [&](const uint64_t (&v)[K]) {
#pragma unroll
    for (int k = 0; k < K; ++k) {
      if ((pending & (1u << k)) && ll_flag(v[k]) == flag) {
        dst[k * kConsumerThreads + tid] = ll_value(v[k]);
        pending &= ~(1u << k);
      }
    }
  };
  Waiter w;
  while (pending) {
    issue(v0);
    check(v0);
    if (!pending) break;
    if (!w.keep_going(c, site)) break;
    if (c.poll_backoff_ns) __nanosleep(c.poll_backoff_ns);
  }
  consumer_sync();
}

// ------------------------------------------------------------- argmax
__device__ __forceinline__ bool arg_better(unsigned ka, int ia, unsigned kb, int ib) {
  return ka > kb || (ka == kb && ia < ib);
}

// Poll every CTA's (key, index) pair for epoch `flag`; all consumer threads
// return the grid-wide argmax (largest logit, lowest index on ties).
__device__ int read_argmax(Ctx &c, unsigned flag, int b = 0) {
  const int tid = threadIdx.x;
  unsigned key = 0;
  int idx = 0x7fffffff;
  if (tid < c.ncta && *c.abort_flag == 0) {
    Waiter w;
    while (true) {
      uint64_t a, bw;
      ll_load2(c.wArg + (size_t)b * kWordsArg + 2 * tid, a, bw);
      if (ll_flag(a) == flag && ll_flag(bw) == flag) {
        key = (unsigned)(a & 0xffffffffu);
        idx = (int)(bw & 0xffffffffu);
        break;
      }
      if (!w.keep_going(c, kSiteArg)) break;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned k2 = __shfl_xor_sync(0xffffffffu, key, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
    if (arg_better(k2, i2, key, idx)) {
      key = k2;
      idx = i2;
    }
  }
  const int warp = tid >> 5, lane = tid & 31;
  __shared__ unsigned s_key[kConsumerWarps];
  __shared__ int s_idx[kConsumerWarps];
  if (lane == 0) {
    s_key[warp] = key;
    s_idx[warp] = idx;
  }
  consumer_sync();
  unsigned bk = s_key[0];
  int bi = s_idx[0];
#pragma unroll
  for (int q = 1; q < kConsumerWarps; ++q) {
    if (arg_better(s_key[q], s_idx[q], bk, bi)) {
      bk = s_key[q];
      bi = s_idx[q];
    }
  }
  consumer_sync();  // s_key/s_idx reusable afterwards
  if (bi < 0 || bi >= kVocab) bi = 0;
  return bi;
}

// ------------------------------------------------------------- producer
// NB: sequences of the batched instance (1 = the single-sequence kernel).
template <bool kFeat, int NB = 1>
struct Producer {
  Ctx &c;
  const Params &p;
  uint64_t pol;
  uint32_t tile = 0;
  bool alive = true;
  int cur_step = 0;  // decode step the tiles being issued belong to

  __device__ Producer(Ctx &c_, const Params &p_) : c(c_), p(p_) { pol = l2_policy_evict_first(); }

  // Reserve the next ring slot for `bytes`; nullptr if the CTA is aborting.
  __device__ uint8_t *begin(unsigned bytes) {
    const int slot = tile % kNumSlots;
    const unsigned use = tile / kNumSlots;
    if (use > 0) {
      Waiter w;
      while (!mbar_try_wait(&c.empty[slot], (use & 1u) ^ 1u)) {
        // the consumers stopped (EOS) before the step this tile belongs to:
        // its slot will not be released, stop issuing
        if (*c.stop_step <= cur_step || !w.keep_going(c, kSiteEmpty)) {
          alive = false;
          return nullptr;
        }
      }
    }
    if (*c.abort_flag) {
      alive = false;
      return nullptr;
    }
    mbar_arrive_expect_tx(&c.full[slot], bytes);
    if (c.trace) {
      const uint32_t k = tile - c.trace_tile0;
      if (k < (uint32_t)kTraceTiles) c.trace[kTraceTileBase + 2 * kTraceTiles + k] = trace_now(c);
    }
    return c.ring + slot * kSlotBytes;
  }
  __device__ __forceinline__ uint64_t *bar() { return &c.full[tile % kNumSlots]; }

  // Part j (of kLmPrefetchLayers) of the L2 prefetch of this CTA's first
  // kLmPrefetchTiles LM-head tiles.
  __device__ void lm_prefetch(int j) {
    const Range r = lm_rows(c.cta, c.ncta);
    const int per = (kLmPrefetchTiles + kLmPrefetchLayers - 1) / kLmPrefetchLayers;
    const uint64_t keep = l2_policy_evict_last();
    for (int t = j * per; t < min(kLmPrefetchTiles, (j + 1) * per); ++t) {
      const int r0 = r.begin + t * kLMTileRows;
      const int n = min(kLMTileRows, r.end - r0);
      if (n <= 0) break;
      bulk_prefetch_l2(reinterpret_cast<const uint8_t *>(p.lm_head) + (size_t)r0 * (kHidden * 2),
                       (unsigned)(n * kHidden * 2), keep);
    }
  }

  // Rows of `mat` in tiles of tile_rows; row k of a tile lands at
  // k * dst_pitch (one copy when the rows are contiguous in the tile).
  __device__ void rows(const __nv_bfloat16 *mat, int row_bytes, Range r, int tile_rows, int dst_pitch) {
    for (int r0 = r.begin; r0 < r.end && alive; r0 += tile_rows) {
      const int n = min(tile_rows, r.end - r0);
      uint8_t *dst = begin((unsigned)(n * row_bytes));
      if (!dst) return;
      const uint8_t *src = reinterpret_cast<const uint8_t *>(mat) + (size_t)r0 * row_bytes;
      if (dst_pitch == row_bytes) {
        bulk_g2s(dst, src, (unsigned)(n * row_bytes), bar(), pol);
      } else {
        for (int k = 0; k < n; ++k)
          bulk_g2s(dst + (size_t)k * dst_pitch, src + (size_t)k * row_bytes, (unsigned)row_bytes, bar(), pol);
      }
      ++tile;
    }
  }

  __device__ void qkv(const LDGLayerWeights &w, Range r) {
    for (int r0 = r.begin; r0 < r.end && alive; r0 += kQKVTileRows) {
      const int n = min(kQKVTileRows, r.end - r0);
      uint8_t *dst = begin((unsigned)(n * 2048));
      if (!dst) return;
      // Split [r0, r0+n) at the q|k|v boundaries (rows 2048 and 3072).
      int a = r0;
      while (a < r0 + n) {
        const __nv_bfloat16 *m;
        int seg0, seg1;
        if (a < kQSize) {
          m = (const __nv_bfloat16 *)w.q_proj_weight;
          seg0 = 0;
          seg1 = kQSize;
        } else if (a < kQSize + kKVSize) {
          m = (const __nv_bfloat16 *)w.k_proj_weight;
          seg0 = kQSize;
          seg1 = kQSize + kKVSize;
        } else {
          m = (const __nv_bfloat16 *)w.v_proj_weight;
          seg0 = kQSize + kKVSize;
          seg1 = kQKVRows;
        }
        const int b = min(r0 + n, seg1);
        bulk_g2s(dst + (size_t)(a - r0) * 2048,
                 reinterpret_cast<const uint8_t *>(m) + (size_t)(a - seg0) * 2048,
                 (unsigned)((b - a) * 2048), bar(), pol);
        a = b;
      }
      ++tile;
    }
  }

  __device__ void gate_up(const LDGLayerWeights &w, Range r) {
    for (int r0 = r.begin; r0 < r.end && alive; r0 += kGUTileRows) {
      const int n = min(kGUTileRows, r.end - r0);
      uint8_t *dst = begin((unsigned)(2 * n * 2048));
      if (!dst) return;
      // gate row k at 4096k, up row k at 4096k + 2048: one tensor-core
      // segment pair per output row.
      const uint8_t *g = reinterpret_cast<const uint8_t *>(w.gate_proj_weight) + (size_t)r0 * 2048;
      const uint8_t *u = reinterpret_cast<const uint8_t *>(w.up_proj_weight) + (size_t)r0 * 2048;
      for (int k = 0; k < n; ++k) {
        bulk_g2s(dst + (size_t)k * 4096, g + (size_t)k * 2048, 2048u, bar(), pol);
        bulk_g2s(dst + (size_t)k * 4096 + 2048, u + (size_t)k * 2048, 2048u, bar(), pol);
      }
      ++tile;
    }
  }

  // K/V rows [chunk) of (sequence b, layer, kv head g).  Positions written
  // earlier in this launch are read only after their writer published kv_ready.
  __device__ void kv(int step, int layer, int b, int g, Range ch) {
    if (ch.end <= ch.begin || !alive) return;
    const int start = (NB > 1) ? p.start_pos_b[b] : p.start_pos;
    if (ch.end > start && step > 0) {
      const unsigned e_prev = epoch_of(c, step - 1, layer, p.num_layers);
      const unsigned e_cur = epoch_of(c, step, layer, p.num_layers);
      const unsigned *flag = &c.ctrl->kv_ready[(b * kMaxLayers + layer) * kNumKVHeads + g];
      Waiter w;
      while (true) {
        const unsigned v = ld_acquire_u32(flag);
        if (v == e_prev || v == e_cur) break;
        if (*c.stop_step <= step || !w.keep_going(c, kSiteKVReady)) {
          alive = false;
          return;
        }
      }
      fence_proxy_async_global();
    }
    const size_t head_off = ((size_t)layer * kNumKVHeads + g) * (size_t)p.max_seq_len;
    const size_t seq_off = (NB > 1) ? (size_t)b * (size_t)p.cache_seq_stride : 0;
    for (int j0 = ch.begin; j0 < ch.end && alive; j0 += kKVTilePos) {
      const int n = min(kKVTilePos, ch.end - j0);
      uint8_t *dst = begin((unsigned)(2 * n * kHeadDim * 2));
      if (!dst) return;
      const size_t off = (head_off + j0) * kHeadDim + seq_off;
      bulk_g2s(dst, p.k_cache + off, (unsigned)(n * kHeadDim * 2), bar(), pol);
      bulk_g2s(dst + kKVTileVOffset, p.v_cache + off, (unsigned)(n * kHeadDim * 2), bar(), pol);
      ++tile;
    }
  }

  __device__ void run() {
    const int item = item_of_cta(c.cta, p.splits, NB);
    const int ib = (item >= 0) ? item / (kNumKVHeads * p.splits) : 0;  // sequence of the item
    const int ig = (item >= 0) ? (item / p.splits) % kNumKVHeads : 0;
    for (int t = 0; t < p.num_steps && alive && *c.stop_step > t; ++t) {
      cur_step = t;
      const int pos = ((NB > 1) ? p.start_pos_b[ib] : p.start_pos) + t;
      c.trace = (kFeat && p.trace && t == p.trace_step) ? p.trace + (size_t)c.cta * kTraceStride : nullptr;
      c.trace_tile0 = tile;
      for (int l = 0; l < p.num_layers && alive; ++l) {
        c.cur_layer = l;
        const LDGLayerWeights w = p.layers[l];
        // The layers leave most of the HBM bandwidth unused while the LM head
        // is bound by it: during the last layers the first LM-head tiles of
        // this CTA are requested into L2 (evict-last), so that the LM-head
        // phase reads them from L2.
        if (l >= p.num_layers - kLmPrefetchLayers) lm_prefetch(l - (p.num_layers - kLmPrefetchLayers));
        trace_stamp(c, true, l * 16 + 12);
        qkv(w, qkv_rows(c.cta, c.ncta));
        if (item >= 0) kv(t, l, ib, ig, kv_chunk(pos, item % p.splits, p.splits));
        rows((const __nv_bfloat16 *)w.o_proj_weight, kQSize * 2, o_rows(c.cta, c.ncta), kOTileRows, kQSize * 2);
        gate_up(w, gu_rows(c.cta, c.ncta));
        rows((const __nv_bfloat16 *)w.down_proj_weight, kInter * 2, d_rows(c.cta, c.ncta), kDTileRows,
             kDRowPitch);
        trace_stamp(c, true, l * 16 + 13);
      }
      trace_stamp(c, true, p.num_layers * 16 + 3);
      rows(p.lm_head, kHidden * 2, lm_rows(c.cta, c.ncta), kLMTileRows, kHidden * 2);
      trace_stamp(c, true, p.num_layers * 16 + 4);
    }
    // Drain: the last tile issued into each slot must land before the CTA exits.
    for (int s = 0; s < kNumSlots; ++s) {
      if (tile > (uint32_t)s) {
        const uint32_t last = s + ((tile - 1u - s) / kNumSlots) * kNumSlots;
        const unsigned par = (last / kNumSlots) & 1u;
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&c.full[s], par)) {
          if (global_timer_ns() - t0 > c.timeout_ns) {
            raise_error(c, QMK_ERR_TIMEOUT, kSiteFull);
            break;
          }
        }
      }
    }
  }
};

// ------------------------------------------------------------- consumer
// kFeat: the feature instance of the kernel (sampling with temperature and
// top-k, timeline trace, store/poll tuning knobs).  The greedy instance
// carries none of that code: the kernel cycles through nearly all of its code
// every layer, and on B200 every KB less in that loop is measurable (the
// optional features cost ~17 us/token when compiled into the common path).
template <bool kFeat, int NB = 1>
struct Consumer {
  Ctx &c;
  const Params &p;
  uint8_t *smem;
  float *sX, *sA, *sAtt, *sU, *sXW;
  // Batched instance: the sequence a phase is working on, and per sequence
  // the residual inputs of this CTA's O rows (from X) and down rows (from A).
  int cur_b = 0;
  float *sResO, *sResD;  // [kMaxSeqs][kMaxResRows]
  float *sPart;  // [2][16][kKsplitGroupRows] K-split partial sums
  unsigned kpart_seq = 0;  // K-split phases run so far (selects the partials buffer)
  float *red_x, *red_a, *red_lm, *red_e;  // block-reduction slots, one per call site
  uint32_t tile = 0;
  unsigned mma_seq = 0;      // tensor-core units consumed (buffer = seq % kTmemBufs)
  float lm_best = -INFINITY;  // LM head: this thread's best logit and row
  int lm_best_i = 0x7fffffff;
  float *lm_logits = nullptr;
  int lm_pos = 0;             // LM head: cache position of the step (sampling key)
  unsigned mma_issued = 0;   // issuer threads: 1 + the last unit this thread issued
  bool tc_prewaited = false; // issuer threads: the next phase's first unit needs no waits
  NormPairs nw_pref;         // RMSNorm weights of the next normalized GEMV input
  int warp, lane, tid;
  uint64_t kv_written = 0;  // layers whose new K/V row this CTA wrote this step

  __device__ Consumer(Ctx &c_, const Params &p_, uint8_t *smem_) : c(c_), p(p_), smem(smem_) {
    sX = reinterpret_cast<float *>(smem + kSmX);
    sA = reinterpret_cast<float *>(smem + kSmA);
    sAtt = reinterpret_cast<float *>(smem + kSmAtt);
    sU = reinterpret_cast<float *>(smem + kSmU);
    sXW = reinterpret_cast<float *>(smem + kSmXW);
    sPart = reinterpret_cast<float *>(smem + kSmMisc + kMiscPart);
    sResO = reinterpret_cast<float *>(smem + kSmMisc + kMiscRes);
    sResD = sResO + kMaxSeqs * kMaxResRows;
    float *red = reinterpret_cast<float *>(smem + kSmMisc + kMiscRed);
    red_x = red;
    red_a = red + 16;
    red_lm = red + 32;
    red_e = red + 48;
    tid = threadIdx.x;
    warp = tid >> 5;
    lane = tid & 31;
  }

  __device__ __forceinline__ bool live() const { return *c.abort_flag == 0; }

  // Slots (N / 16) of a GEMV kind.
  __device__ static int tc_slots(int kind) { return (kind == kTcHalf) ? 2 : (kind == kTcQuarter) ? 3 : 1; }

  // Issue the 4 MMAs of M block hp of ring tile `tl` (tensor-core unit
  // number seq) into TMEM buffer seq % kTmemBufs, against the B operand at
  // bop with S slots.  Layout of A, B and D: see the GEMV section above.
  // Called by a whole issuer warp: lane 0 waits (unless `waited`: its
  // pre-wait already did), one elected lane issues.  A K step of 16 moves
  // both descriptors' start address by 32 bytes (2 in the 16-byte field).
  __device__ bool tc_issue_unit(uint32_t tl, int hp, unsigned seq, const uint8_t *bop, int S, bool waited) {
    const uint32_t idesc = mma_idesc_bf16(128, 16 * S);
    const unsigned b = seq % kTmemBufs;
    bool ok = true;
    if (lane == 0 && !waited) ok = tc_unit_waits(tl, seq);
    if (!__shfl_sync(0xffffffffu, (int)ok, 0)) return false;
    tc_fence_after_sync();
    const uint64_t ad = smem_desc_sw128(smem_addr(slot_ptr(c, tl)) + 1024u * (uint32_t)hp, 2048u);
    const uint64_t bd = smem_desc_sw128(smem_addr(bop) + 2048u * (uint32_t)(S * hp), 1024u);
    const uint32_t d = c.tmem + (uint32_t)kTmemBufCols * b;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) tc_mma_bf16_warp(d, ad + 2u * kk, bd + 2u * kk, idesc, kk > 0);
    tc_commit_warp(&c.mma_bar[b]);
    mma_issued = seq + 1u;
    return true;
  }

  // What a unit needs before its MMAs: its TMEM buffer read out by the
  // readers of the unit that used it before, and its ring tile landed.
  __device__ bool tc_unit_waits(uint32_t tl, unsigned seq) {
    if (seq >= (unsigned)kTmemBufs) {
      const unsigned par = ((seq / kTmemBufs) - 1u) & 1u;
      Waiter w;
      while (!mbar_try_wait(&c.tmem_free[seq % kTmemBufs], par))
        if (!w.keep_going(c, kSiteMma)) return false;
    }
    return wait_full_one(c, tl);
  }

  // Issuers, before the phase's input is staged: the waits of the first unit
  // each issues, so that its MMAs can start as soon as the B operand is ready.
  __device__ void tc_prewait(int r0, int r1, int tile_rows) {
    tc_prewaited = false;
    if (warp >= 4 && lane == 0 && live()) {
      const int u = warp - 4;
      const int ntiles = (r1 - r0 + tile_rows - 1) / tile_rows;
      if (u < 2 * ntiles) tc_prewaited = tc_unit_waits(tile + (uint32_t)(u >> 1), mma_seq + (unsigned)u);
    }
  }

  // Reader side: wait (bounded) for tensor-core unit seq.
  __device__ bool wait_unit(unsigned seq) {
    const unsigned par = (seq / kTmemBufs) & 1u;
    Waiter w;
    while (!mbar_try_wait(&c.mma_bar[seq % kTmemBufs], par))
      if (!w.keep_going(c, kSiteMma)) return false;
    return true;
  }

  // One GEMV phase on the tensor cores (see tc_phase).
  struct TcJob {
    int kind;       // TcKind: tile layout
    int out;        // TcOut: what the rows produce
    int r0, r1;     // this CTA's rows
    int tile_rows;  // rows per ring tile
    float scale;    // 1/rms of a normalized input (1 otherwise)
    unsigned E;     // epoch of the output words
  };

  // Row `row` of a phase, value v (and v2: the up projection of kOutGU).
  __device__ void tc_emit(const TcJob &job, int row, float v, float v2) {
    switch (job.out) {
      case kOutQKV:
        put(c.wQKV + (NB > 1 ? (size_t)cur_b * kWordsQKV : 0) + row, ll_pack(v * job.scale, job.E));
        break;
      case kOutO: {
        const float res = (NB > 1) ? sResO[cur_b * kMaxResRows + (row - job.r0)] : sX[row];
        put(c.wA + (NB > 1 ? (size_t)cur_b * kWordsA : 0) + row, ll_pack(v + res, job.E));
        break;
      }
      case kOutGU: {
        const float gs = v * job.scale, us = v2 * job.scale;
        const float silu = gs * fast_rcp(1.0f + fast_exp2(-gs * kLog2e));
        put(c.wM + (NB > 1 ? (size_t)cur_b * kWordsM : 0) + row, ll_pack(silu * us, job.E));
        break;
      }
      case kOutDown: {
        const float res = (NB > 1) ? sResD[cur_b * kMaxResRows + (row - job.r0)] : sA[row];
        put(c.wX + (NB > 1 ? (size_t)cur_b * kWordsX : 0) + row, ll_pack(v + res, job.E));
        break;
      }
      default: {  // kOutLM
        const float y = v * job.scale;
        if constexpr (kFeat) {
          if (p.top_k > 0) {  // top-k sampling: the selection runs on all rows afterwards
            sU[kHidden + (row - job.r0)] = y;  // after the LM-head B operand (sU[0, 1024))
            if (lm_logits) lm_logits[row] = y;
            break;
          }
        }
        // greedy: the logit; sampling: logit / T + Gumbel noise
        const float key = (kFeat && p.inv_temp > 0.f) ? fmaf(y, p.inv_temp, gumbel_noise(p.seed, lm_pos, row)) : y;
        if (key > lm_best || (key == lm_best && row < lm_best_i)) {
          lm_best = key;
          lm_best_i = row;
        }
        if (lm_logits) lm_logits[row] = y;
        break;
      }
    }
  }

  // GEMV phase over the ring tiles of rows [r0, r1) on the tensor cores.
  // A unit is one M block (4 MMAs); warps 4-6 issue the units round-robin
  // (one issuer is limited by the issue latency of tcgen05.mma), up to
  // kTmemBufs units in flight; warps 0-3 read both units
  // of a tile (one TMEM lane each), add the diagonal entries of every output
  // row with warp shuffles and emit each row from one lane.
  //   kTcRow     K = 1024, 16 rows
  //   kTcGU      K = 1024, tile rows 2k (gate) and 2k+1 (up) of output row
  //              k (8 rows)
  //   kTcHalf    K = 2048, 8 rows
  //   kTcQuarter K = 3072, 4 rows at an 8 KB pitch
  __device__ __forceinline__ void tc_phase(const TcJob &job, const uint8_t *bop) {
    const int S = tc_slots(job.kind);
    const int ntiles = (job.r1 - job.r0 + job.tile_rows - 1) / job.tile_rows;
    constexpr int kIssuers = kConsumerWarps - 4;
    const unsigned seq0 = mma_seq;
    const int nunits = 2 * ntiles;
    if (warp >= 4) {
      bool ok = live();
      for (int u = warp - 4; u < nunits && ok; u += kIssuers)
        ok = tc_issue_unit(tile + (uint32_t)(u >> 1), u & 1, seq0 + (unsigned)u, bop, S,
                           u == warp - 4 && tc_prewaited);
      tc_prewaited = false;
    }
    if (warp < 4) {
      const int q = lane & 7;
      const int j = (32 * warp + lane) >> 3;  // segment of this lane
      const int slot = (job.kind == kTcHalf) ? (j & 1) : (job.kind == kTcQuarter) ? (j & 3) : 0;
      const bool valid = slot < S;            // K = 3072: quarter 3 of a row is unused
      for (int t = 0; t < ntiles; ++t) {
        const unsigned seq = seq0 + 2u * (unsigned)t;
        bool got = live() && wait_unit(seq) && wait_unit(seq + 1u);
        got = __all_sync(0xffffffffu, got);
        const uint32_t tk = tile + (uint32_t)t - c.trace_tile0;
        const bool tstamp = c.trace && tid == 0 && tk < (uint32_t)kTraceTiles;
        if (got && tid == 0) {
          // both units' MMAs have read the tile: hand the ring slot back
          if (tstamp) c.trace[kTraceTileBase + 3 * kTraceTiles + tk] = trace_now(c);
          mbar_arrive_cnt(&c.empty[(tile + (uint32_t)t) % kNumSlots], kConsumerWarps);
        }
        __syncwarp();
        float v = 0.f;
        if (got) {
          tc_fence_after_sync();
#pragma unroll
          for (int hp = 0; hp < 2; ++hp) {
            const uint32_t taddr =
                c.tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)kTmemBufCols * ((seq + (unsigned)hp) % kTmemBufs);
            v += (S == 1) ? tc_read<1>(taddr, slot, q) : (S == 2) ? tc_read<2>(taddr, slot, q) : tc_read<3>(taddr, slot, q);
          }
          if (!valid) v = 0.f;
        }
        tc_fence_before_sync();
        if (tstamp) c.trace[kTraceTileBase + 4 * kTraceTiles + tk] = trace_now(c);
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        if (job.kind == kTcHalf || job.kind == kTcQuarter) v += __shfl_xor_sync(0xffffffffu, v, 8);
        if (job.kind == kTcQuarter) v += __shfl_xor_sync(0xffffffffu, v, 16);
        const float up = __shfl_down_sync(0xffffffffu, v, 8);
        int lrow = -1;
        if (job.kind == kTcRow) {
          if (q == 0) lrow = j;
        } else if (job.kind == kTcQuarter) {
          if (lane == 0) lrow = warp;
        } else if ((lane & 15) == 0) {
          lrow = j >> 1;
        }
        const int row = job.r0 + t * job.tile_rows + lrow;
        if (got && lrow >= 0 && row < job.r1) tc_emit(job, row, v, up);
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&c.tmem_free[seq % kTmemBufs]);
          mbar_arrive(&c.tmem_free[(seq + 1u) % kTmemBufs]);
        }
        if (tstamp) c.trace[kTraceTileBase + 5 * kTraceTiles + tk] = trace_now(c);
      }
    }
    tile += (uint32_t)ntiles;
    mma_seq += (unsigned)nunits;
  }

  // Batched instance: a K = 1024 GEMV phase (kTcRow or kTcGU tiles) of all
  // NB staged inputs on the tensor cores in one pass over the tiles.  The B
  // operand holds the NB inputs side by side (stage_vecs kStageNormFrag:
  // slot b = sequence b, N = 16 NB), so each unit (one M block, 4 MMAs)
  // multiplies its half-tile with every input and D[8j + q][16b + 8g + q]
  // is segment j's partial (part g) for sequence b.  Issuers as in
  // tc_phase; each reader lane loads its TMEM lane's 16 NB columns of both
  // units, adds its 2 NB diagonal entries per sequence, and an 8-lane
  // transposing reduction leaves sequence q >> 1's segment sum in lane q of
  // the segment (q = lane & 7), which emits it scaled by that sequence's
  // 1/rms (`scale`).  Rows as in tc_phase: a tile row per segment (kTcRow),
  // or gate (segment 2k) and up (2k + 1) of output row k (kTcGU).
  __device__ __forceinline__ void tc_phase_nb(const TcJob &job, const uint8_t *bop, const float (&scale)[NB]) {
    static_assert(NB == 4, "one sequence per lane pair of a segment");
    const int ntiles = (job.r1 - job.r0 + job.tile_rows - 1) / job.tile_rows;
    constexpr int kIssuers = kConsumerWarps - 4;
    const unsigned seq0 = mma_seq;
    const int nunits = 2 * ntiles;
    if (warp >= 4) {
      bool ok = live();
      for (int u = warp - 4; u < nunits && ok; u += kIssuers)
        ok = tc_issue_unit(tile + (uint32_t)(u >> 1), u & 1, seq0 + (unsigned)u, bop, NB,
                           u == warp - 4 && tc_prewaited);
      tc_prewaited = false;
    }
    if (warp < 4) {
      const int q = lane & 7;
      const int j = (32 * warp + lane) >> 3;  // segment of this lane
      const int mb = q >> 1;                  // sequence whose sum this lane ends with
      TcJob jb = job;
      jb.scale = (mb == 0) ? scale[0] : (mb == 1) ? scale[1] : (mb == 2) ? scale[2] : scale[3];
      cur_b = mb;
      for (int t = 0; t < ntiles; ++t) {
        const unsigned seq = seq0 + 2u * (unsigned)t;
        bool got = live() && wait_unit(seq) && wait_unit(seq + 1u);
        got = __all_sync(0xffffffffu, got);
        if (got && tid == 0) mbar_arrive_cnt(&c.empty[(tile + (uint32_t)t) % kNumSlots], kConsumerWarps);
        __syncwarp();
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        if (got) {
          tc_fence_after_sync();
#pragma unroll
          for (int hp = 0; hp < 2; ++hp) {
            const uint32_t taddr =
                c.tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)kTmemBufCols * ((seq + (unsigned)hp) % kTmemBufs);
            uint32_t r[32];
#pragma unroll
            for (int h = 0; h < 2; ++h) {  // columns 32h .. 32h + 31: sequences 2h, 2h + 1
              tmem_ld32(taddr + 32u * (uint32_t)h, r);
              v[2 * h] += sel8(r, q) + sel8(r + 8, q);
              v[2 * h + 1] += sel8(r + 16, q) + sel8(r + 24, q);
            }
          }
        }
        tc_fence_before_sync();
        const float sum = reduce4_oct(v);
        const float up = __shfl_down_sync(0xffffffffu, sum, 8);
        int lrow = -1;
        if ((q & 1) == 0) {
          if (job.kind == kTcRow)
            lrow = j;
          else if ((lane & 8) == 0)
            lrow = j >> 1;
        }
        const int row = job.r0 + t * job.tile_rows + lrow;
        if (got && lrow >= 0 && row < job.r1) tc_emit(jb, row, sum, up);
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&c.tmem_free[seq % kTmemBufs]);
          mbar_arrive(&c.tmem_free[(seq + 1u) % kTmemBufs]);
        }
      }
    }
    tile += (uint32_t)ntiles;
    mma_seq += (unsigned)nunits;
  }

  // GEMV phases on the CUDA cores.  The weights of a phase stream through
  // the ring in tiles of tile_rows rows at `pitch` bytes (the layouts of the
  // producer's bulk copies), the input vector x is fp32 in shared memory.
  // Shared-memory bandwidth (128 B per clock) bounds these loops, so every
  // weight byte and, as far as possible, every x byte is read once, with
  // conflict-free accesses: lane l takes elements 4l + 128j + (0..3) of a
  // 1024-element chunk (x as one float4 per j, weights as one 8-byte pair
  // of bf16 pairs per j, a warp reading 256 contiguous bytes per j).

  // The weight tiles of a phase are normally resident before its input
  // arrives (the stream runs a layer ahead), so a phase waits for all of
  // its tiles first and then gives every warp all of its work at once: the
  // loads of several rows are in flight together, which a single warp needs
  // to hide shared-memory latency.  The tiles are released at the end.
  // Wait for the phase's tiles (ntiles <= kNumSlots).  The first pass tests
  // every tile's barrier with independent try_waits, which overlap (a
  // try_wait on a completed phase still costs ~120 cycles here); only tiles
  // not landed yet take the bounded wait loop.
  __device__ __forceinline__ bool wait_tiles(int ntiles) {
    const bool stamp = c.trace && tid == 0 && tile - c.trace_tile0 + (uint32_t)ntiles <= (uint32_t)kTraceTiles;
    uint64_t t0 = 0;
    if (stamp) t0 = trace_now(c);
    unsigned miss = 0;
    bool hit[kNumSlots];
#pragma unroll
    for (int t = 0; t < kNumSlots; ++t) {
      const uint32_t tt = tile + (uint32_t)t;
      hit[t] = (t < ntiles) ? mbar_try_wait(&c.full[tt % kNumSlots], (tt / kNumSlots) & 1u) : true;
    }
#pragma unroll
    for (int t = 0; t < kNumSlots; ++t) miss |= hit[t] ? 0u : (1u << t);
    bool ok = true;
    if (__any_sync(0xffffffffu, miss != 0u)) {
      for (int t = 0; t < ntiles; ++t) ok = wait_full(c, tile + (uint32_t)t) && ok;
    } else if (stamp) {
      // the stamps of wait_full (wait entry, tile seen landed): every tile
      // had landed when the warp first tested it
      for (int t = 0; t < ntiles; ++t) {
        const uint32_t k = tile + (uint32_t)t - c.trace_tile0;
        c.trace[kTraceTileBase + 2 * k] = t0;
        c.trace[kTraceTileBase + 2 * k + 1] = t0;
      }
    }
    return ok;
  }
  // Tiles of a phase over rows [R.begin, R.end) at tile_rows rows per tile.
  static __device__ __forceinline__ int tiles_of(const Range &R, int tile_rows) {
    return (R.end - R.begin + tile_rows - 1) / tile_rows;
  }

  // Release the phase's tiles: one arrive per tile from lane 0 once the warp
  // has finished reading them.
  __device__ __forceinline__ void release_tiles(int ntiles, bool ok) {
    if (c.trace && tid == 0) {
      for (int t = 0; t < ntiles; ++t) {
        const uint32_t k = tile + (uint32_t)t - c.trace_tile0;
        if (k < (uint32_t)kTraceTiles) c.trace[kTraceTileBase + 3 * kTraceTiles + k] = trace_now(c);
      }
    }
    __syncwarp();
    if (ok && lane == 0) {
      for (int t = 0; t < ntiles; ++t) mbar_arrive(&c.empty[(tile + (uint32_t)t) % kNumSlots]);
    }
    tile += (uint32_t)ntiles;
  }
  // Address of byte `off` of row i of the phase (tiles of tile_rows rows at
  // `pitch` bytes, consecutive ring slots).
  __device__ __forceinline__ const uint8_t *row_ptr(int i, int tile_rows, int pitch, int off) const {
    return slot_ptr(c, tile + (uint32_t)(i / tile_rows)) + (size_t)(i % tile_rows) * pitch + off;
  }

  // Row split (q|k|v, gate/up: K = 1024, many rows): phase row i is computed
  // by warp i % kConsumerWarps, MR rows of a warp at a time; the warp adds
  // the lanes' partial sums with a butterfly and lane 0 emits.  kOutGU: a
  // gate row and, 2048 bytes further, an up row per output row.  No barrier
  // between the warps.
  template <int OUT, int MR>
  __device__ void fma_rows_phase(bool ok, const float *x, int r0, int r1, int tile_rows, int pitch, float scale,
                                 unsigned E, bool release = true) {
    constexpr bool kGU = (OUT == kOutGU);
    static_assert(MR >= 1 && MR <= 4, "rows per warp batch");
    const TcJob job{kTcRow, OUT, r0, r1, tile_rows, scale, E};
    const int n = r1 - r0;
    const int ntiles = (n + tile_rows - 1) / tile_rows;
    float4 xv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) xv[j] = reinterpret_cast<const float4 *>(x)[lane + 32 * j];
    for (int i0 = warp; ok && i0 < n; i0 += kConsumerWarps * MR) {
      // rows i0 + 7r of this batch; rows past the end repeat row i0 (no
      // branch inside the loop, so the rows' FMA chains interleave)
      const uint8_t *rp[MR];
#pragma unroll
      for (int r = 0; r < MR; ++r) {
        const int i = i0 + kConsumerWarps * r;
        rp[r] = row_ptr(i < n ? i : i0, tile_rows, pitch, 8 * lane);
      }
      float s[MR][kGU ? 8 : 4];
#pragma unroll
      for (int r = 0; r < MR; ++r)
#pragma unroll
        for (int a = 0; a < (kGU ? 8 : 4); ++a) s[r][a] = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        uint2 w[MR], u[kGU ? MR : 1];
#pragma unroll
        for (int r = 0; r < MR; ++r) {
          w[r] = *reinterpret_cast<const uint2 *>(rp[r] + 256 * j);
          if (kGU) u[kGU ? r : 0] = *reinterpret_cast<const uint2 *>(rp[r] + 2048 + 256 * j);
        }
#pragma unroll
        for (int r = 0; r < MR; ++r) {
          s[r][0] = fmaf(xv[j].x, bf_lo(w[r].x), s[r][0]);
          s[r][1] = fmaf(xv[j].y, bf_hi(w[r].x), s[r][1]);
          s[r][2] = fmaf(xv[j].z, bf_lo(w[r].y), s[r][2]);
          s[r][3] = fmaf(xv[j].w, bf_hi(w[r].y), s[r][3]);
          if (kGU) {
            const uint2 q = u[kGU ? r : 0];
            s[r][kGU ? 4 : 0] = fmaf(xv[j].x, bf_lo(q.x), s[r][kGU ? 4 : 0]);
            s[r][kGU ? 5 : 1] = fmaf(xv[j].y, bf_hi(q.x), s[r][kGU ? 5 : 1]);
            s[r][kGU ? 6 : 2] = fmaf(xv[j].z, bf_lo(q.y), s[r][kGU ? 6 : 2]);
            s[r][kGU ? 7 : 3] = fmaf(xv[j].w, bf_hi(q.y), s[r][kGU ? 7 : 3]);
          }
        }
      }
      float v[4], v2[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        v[r] = v2[r] = 0.f;
        if (r < MR) {
          v[r] = (s[r][0] + s[r][1]) + (s[r][2] + s[r][3]);
          v2[r] = kGU ? (s[r][kGU ? 4 : 0] + s[r][kGU ? 5 : 1]) + (s[r][kGU ? 6 : 2] + s[r][kGU ? 7 : 3]) : 0.f;
        }
      }
      // Transposing butterfly: after it lane l holds the warp sum of row
      // 2 ((l >> 4) & 1) + ((l >> 3) & 1) of the batch (6 shuffles per value
      // instead of 5 per row), and lanes 0, 8, 16, 24 emit in parallel.
      const int rr = 2 * ((lane >> 4) & 1) + ((lane >> 3) & 1);
      const float sum = reduce4_transpose(v);
      const float sum2 = kGU ? reduce4_transpose(v2) : 0.f;
      const int i = i0 + kConsumerWarps * rr;
      if ((lane & 7) == 0 && rr < MR && i < n) tc_emit(job, r0 + i, sum, sum2);
    }
    if (release) release_tiles(ntiles, ok);
  }

  // K split (O: K = 2048, down: K = 3072; about as many rows per CTA as
  // warps): the 128-element blocks of K are dealt to the warps round-robin
  // and every warp multiplies its blocks of all rows, so x and the weights
  // are read once per CTA.  Rows go through registers in batches of
  // kKsplitRows; the warps' partial row sums of up to kKsplitGroupRows rows
  // meet in shared memory (double-buffered) behind one consumer barrier, and
  // thread r then adds row r's partials in warp order (deterministic) and
  // emits it.  148 CTAs: 6-7 rows, one barrier per phase.
  template <int KC, int OUT>
  __device__ void fma_ksplit_phase(bool ok, const float *x, int r0, int r1, int tile_rows, int pitch, unsigned E,
                                   bool release = true) {
    constexpr int kBlocks = 8 * KC;  // 128-element blocks per row
    constexpr int kMine = (kBlocks + kConsumerWarps - 1) / kConsumerWarps;
    constexpr int RB = kKsplitRows;
    constexpr int RG = kKsplitGroupRows;
    static_assert(RB == 4 && RG % RB == 0, "the transposing reduction handles 4 rows");
    const TcJob job{kTcRow, OUT, r0, r1, tile_rows, 1.f, E};
    const int n = r1 - r0;
    const int ntiles = (n + tile_rows - 1) / tile_rows;
    float4 xv[kMine];
#pragma unroll
    for (int q = 0; q < kMine; ++q) {
      const int b = warp + kConsumerWarps * q;
      xv[q] = (b < kBlocks) ? reinterpret_cast<const float4 *>(x)[lane + 32 * b] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int g0 = 0; g0 < n; g0 += RG) {  // every warp runs every group (barrier inside)
      float *part = sPart + (kpart_seq++ & 1) * (16 * RG);
      const int gn = min(RG, n - g0);
      for (int b0 = 0; b0 < gn; b0 += RB) {
        const int i0 = g0 + b0;
        float v[RB];
#pragma unroll
        for (int r = 0; r < RB; ++r) v[r] = 0.f;
        if (ok) {
          uint2 w[RB][kMine];
#pragma unroll
          for (int r = 0; r < RB; ++r) {
            if (i0 + r < n) {
              const uint8_t *rp = row_ptr(i0 + r, tile_rows, pitch, 8 * lane);
#pragma unroll
              for (int q = 0; q < kMine; ++q) {
                const int b = warp + kConsumerWarps * q;
                if (b < kBlocks) w[r][q] = *reinterpret_cast<const uint2 *>(rp + 256 * b);
              }
            }
          }
#pragma unroll
          for (int r = 0; r < RB; ++r) {
            if (i0 + r < n) {
              float s0 = 0.f, s1 = 0.f;
#pragma unroll
              for (int q = 0; q < kMine; ++q)
                if (warp + kConsumerWarps * q < kBlocks) dot4(s0, s1, w[r][q], xv[q]);
              v[r] = s0 + s1;
            }
          }
        }
        const float wsum = reduce4_transpose(v);
        if ((lane & 7) == 0) part[warp * RG + b0 + 2 * ((lane >> 4) & 1) + ((lane >> 3) & 1)] = wsum;
      }
      consumer_sync();
      if (tid < gn && ok) {
        float sum = 0.f;
#pragma unroll
        for (int q = 0; q < kConsumerWarps; ++q) sum += part[q * RG + tid];
        tc_emit(job, r0 + g0 + tid, sum, 0.f);
      }
    }
    if (release) release_tiles(ntiles, ok);
  }

  // Issuer threads: wait (bounded) for the last MMAs they issued, so that
  // TMEM can be freed (normally they were consumed already).
  __device__ void drain_mma() {
    if (mma_issued > 0u) {
      const unsigned seq = mma_issued - 1u;
      const unsigned par = (seq / kTmemBufs) & 1u;
      const uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(&c.mma_bar[seq % kTmemBufs], par)) {
        if (global_timer_ns() - t0 > c.timeout_ns) break;
      }
    }
  }

  // Store of one dataflow word.  Default: an L2 atomic max (red.max.u64) --
  // plain stores could sit in the SM's write path for microseconds before
  // other SMs saw them, atomics are performed at L2 right away.  Tuning bits
  // 0-1 of QmkRunArgs.tuning select alternatives for measurement:
  // 1 st.relaxed.gpu, 2 st.relaxed.gpu + fence at the end of the phase,
  // 3 atom.exch.b64.
  __device__ __forceinline__ void put(uint64_t *q, uint64_t w) const {
    switch (c.tuning & 3u) {
      case 0: ll_store_redmax(q, w); break;
      case 3: ll_store_exch(q, w); break;
      default: ll_store(q, w); break;
    }
  }
  __device__ __forceinline__ void flush() const {
    if ((c.tuning & 3u) == 2u) __threadfence();
  }

  // P1: RMSNorm(x) then q|k|v rows of this CTA.
  // x_flag: epoch of the X words to stage, or 0 when sX already holds the
  // layer input (the embedding row of layer 0) and x_ss its sum of squares.
  __device__ void phase_qkv(const LDGLayerWeights &w, unsigned E, int l, unsigned x_flag, float x_ss) {
    const NormPairs nw = nw_pref;  // fetched one phase ahead
    const Range R = qkv_rows(c.cta, c.ncta);
    // The weight tiles have normally landed long before the input: their
    // barrier tests (strong shared-memory operations, ~120+ cycles each)
    // run before the dataflow wait instead of after it, likewise below.
    const bool tiles = wait_tiles(tiles_of(R, kQKVTileRows));
    if (x_flag) {
      x_ss = stage_vec<kHidden, kStageNorm>(c, sX, reinterpret_cast<uint8_t *>(sXW), c.wX, x_flag, kSiteX, red_x, nw);
    } else {
      build_norm_xw(sXW, sX, nw, tid);
      consumer_sync();
    }
    trace_stamp(c, tid == 0, l * 16 + 0);
    fma_rows_phase<kOutQKV, 4>(tiles, sXW, R.begin, R.end, kQKVTileRows, 2048, rsqrtf(x_ss / (float)kHidden + kRmsEps), E);
    flush();
    trace_stamp(c, tid == 0, l * 16 + 1);
  }

  // P2: one split-KV attention item for KV head g (q heads 2g, 2g+1).
  __device__ void phase_attention(const LDGLayerWeights &w, int layer, int step, unsigned E) {
    const int item = item_of_cta(c.cta, p.splits, NB);
    if (item < 0) return;
    const int g = (item / p.splits) % kNumKVHeads, s = item % p.splits;
    const int b = (NB > 1) ? item / (kNumKVHeads * p.splits) : 0;  // sequence
    const bool last = (s == p.splits - 1);
    const int pos = ((NB > 1) ? p.start_pos_b[b] : p.start_pos) + step;
    const Range ch = kv_chunk(pos, s, p.splits);
    float *sQ = sU + kUQ;
    float *sPW = sU + kUPW;

    // Operands that do not depend on this step's activations are fetched
    // before the dataflow wait: QK-norm weights and the position's cos/sin.
    const int d0 = 4 * lane;
    const bool rope_warp = warp < 2 || (warp == 2 && last);
    uint2 nwv = make_uint2(0u, 0u), cvv = make_uint2(0u, 0u), svv = make_uint2(0u, 0u);
    if (rope_warp) {
      const __nv_bfloat16 *nw = (const __nv_bfloat16 *)((warp < 2) ? w.q_norm_weight : w.k_norm_weight);
      nwv = __ldg(reinterpret_cast<const uint2 *>(nw + d0));
      cvv = __ldg(reinterpret_cast<const uint2 *>(p.cos_t + (size_t)pos * kHeadDim + d0));
      svv = __ldg(reinterpret_cast<const uint2 *>(p.sin_t + (size_t)pos * kHeadDim + d0));
    }

    // q rows [256g, 256g+256), k rows 2048+128g.., v rows 3072+128g.. -> sU[0..512)
    stage_list<(512 + kConsumerThreads - 1) / kConsumerThreads>(
        c, sU, 512,
        [&](int i) -> const uint64_t * {
          const int row = (i < 256) ? (g * 256 + i)
                                    : (i < 384) ? (kQSize + g * 128 + (i - 256))
                                                : (kQSize + kKVSize + g * 128 + (i - 384));
          return c.wQKV + (NB > 1 ? (size_t)b * kWordsQKV : 0) + row;
        },
        E, kSiteQKV);
    trace_stamp(c, tid == 0, layer * 16 + 2);

    // Per-head RMSNorm + RoPE (rotate-half).  Lane l holds dims 4l..4l+3; the
    // rotation partner dims (d +- 64) sit in lane l ^ 16.
    if (rope_warp) {
      float *vec = (warp < 2) ? (sQ + warp * kHeadDim) : (sU + kUK);
      const float nwf[4] = {bf_lo(nwv.x), bf_hi(nwv.x), bf_lo(nwv.y), bf_hi(nwv.y)};
      const float cvf[4] = {bf_lo(cvv.x), bf_hi(cvv.x), bf_lo(cvv.y), bf_hi(cvv.y)};
      const float svf[4] = {bf_lo(svv.x), bf_hi(svv.x), bf_lo(svv.y), bf_hi(svv.y)};
      float x[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) x[e] = vec[d0 + e];
      float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
      ss = warp_sum(ss);
      const float r = rsqrtf(ss / (float)kHeadDim + kRmsEps);
#pragma unroll
      for (int e = 0; e < 4; ++e) x[e] = (x[e] * r) * nwf[e];
      float y[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float partner = __shfl_xor_sync(0xffffffffu, x[e], 16);
        y[e] = (lane < 16) ? (x[e] * cvf[e] - partner * svf[e]) : (x[e] * cvf[e] + partner * svf[e]);
      }
      if (warp < 2) {
        const float qs = p.attn_scale * kLog2e;  // scores in log2 units
#pragma unroll
        for (int e = 0; e < 4; ++e) vec[d0 + e] = y[e] * qs;
      } else {
        // New K/V row of this position, bf16: into the cache and, in the
        // cache's row format, into smem for this step's softmax.
        const size_t off = (((size_t)layer * kNumKVHeads + g) * (size_t)p.max_seq_len + pos) * kHeadDim + d0 +
                           (NB > 1 ? (size_t)b * (size_t)p.cache_seq_stride : 0);
        unsigned kbits[4], vbits[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          kbits[e] = __bfloat16_as_ushort(__float2bfloat16(y[e]));
          vbits[e] = __bfloat16_as_ushort(__float2bfloat16(sU[kUV + d0 + e]));
        }
        const uint2 kw = make_uint2(kbits[0] | (kbits[1] << 16), kbits[2] | (kbits[3] << 16));
        const uint2 vw = make_uint2(vbits[0] | (vbits[1] << 16), vbits[2] | (vbits[3] << 16));
        reinterpret_cast<uint2 *>(sU + kUKn)[lane] = kw;
        reinterpret_cast<uint2 *>(sU + kUVn)[lane] = vw;
        *reinterpret_cast<uint2 *>(p.k_cache + off) = kw;
        *reinterpret_cast<uint2 *>(p.v_cache + off) = vw;
      }
    }
    consumer_sync();
    // The new K/V row is published (kv_ready) at the start of the LM-head
    // phase, off the critical path: only the next step's producers read it.
    if (last) kv_written |= 1ull << layer;

    // Online softmax over cache positions.  Group gq = lane / 8 of a warp
    // takes one position per step; lane r8 = lane % 8 of the group holds dims
    // [8 r8, 8 r8 + 8) and [64 + 8 r8, 64 + 8 r8 + 8) of both q heads
    // (16-byte shared-memory reads, one 128-byte line per 8 lanes), so a
    // score is 16 FMAs per head and a 3-level butterfly.  Of a tile, warp w
    // takes positions 28 t + 4 w + gq (t < kSteps) and moves its running max
    // once; the four groups share that max, so their sums add without
    // rescaling at the end.
    const int gq = lane >> 3, r8 = lane & 7;
    float qv[2][16];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float4 *qa = reinterpret_cast<const float4 *>(sQ + h * kHeadDim + 8 * r8);
      const float4 *qb = reinterpret_cast<const float4 *>(sQ + h * kHeadDim + 64 + 8 * r8);
      const float4 v4[4] = {qa[0], qa[1], qb[0], qb[1]};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        qv[h][4 * k + 0] = v4[k].x;
        qv[h][4 * k + 1] = v4[k].y;
        qv[h][4 * k + 2] = v4[k].z;
        qv[h][4 * k + 3] = v4[k].w;
      }
    }
    float mrun[2] = {-INFINITY, -INFINITY}, lrun[2] = {0.f, 0.f};
    float oacc[2][16];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int e = 0; e < 16; ++e) oacc[h][e] = 0.f;
    constexpr int kStride = 4 * kConsumerWarps;
    constexpr int kSteps = (kKVTilePos + kStride - 1) / kStride;
    // Rows j < n: K at kt + 256 j, V at vt + 256 j (bf16, 128 dims each).
    auto absorb = [&](const uint8_t *kt, const uint8_t *vt, int n) {
      if (4 * warp >= n) return;  // warp-uniform: no position of this warp
      int jr[kSteps];
      bool ok[kSteps];
      float s[kSteps][2];
#pragma unroll
      for (int t = 0; t < kSteps; ++t) {
        const int j = kStride * t + 4 * warp + gq;
        ok[t] = j < n;
        jr[t] = ok[t] ? j : 4 * warp;
        const uint8_t *row = kt + (size_t)jr[t] * (kHeadDim * 2) + 16 * r8;
        const uint4 a = *reinterpret_cast<const uint4 *>(row);
        const uint4 b = *reinterpret_cast<const uint4 *>(row + kHeadDim);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float *q = qv[h];
          float s0 = q[0] * bf_lo(a.x), s1 = q[1] * bf_hi(a.x);
          s0 = fmaf(q[2], bf_lo(a.y), s0);
          s1 = fmaf(q[3], bf_hi(a.y), s1);
          s0 = fmaf(q[4], bf_lo(a.z), s0);
          s1 = fmaf(q[5], bf_hi(a.z), s1);
          s0 = fmaf(q[6], bf_lo(a.w), s0);
          s1 = fmaf(q[7], bf_hi(a.w), s1);
          s0 = fmaf(q[8], bf_lo(b.x), s0);
          s1 = fmaf(q[9], bf_hi(b.x), s1);
          s0 = fmaf(q[10], bf_lo(b.y), s0);
          s1 = fmaf(q[11], bf_hi(b.y), s1);
          s0 = fmaf(q[12], bf_lo(b.z), s0);
          s1 = fmaf(q[13], bf_hi(b.z), s1);
          s0 = fmaf(q[14], bf_lo(b.w), s0);
          s1 = fmaf(q[15], bf_hi(b.w), s1);
          s[t][h] = s0 + s1;
        }
      }
      uint4 va[kSteps], vb[kSteps];
#pragma unroll
      for (int t = 0; t < kSteps; ++t) {
        const uint8_t *row = vt + (size_t)jr[t] * (kHeadDim * 2) + 16 * r8;
        va[t] = *reinterpret_cast<const uint4 *>(row);
        vb[t] = *reinterpret_cast<const uint4 *>(row + kHeadDim);
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1)
#pragma unroll
        for (int t = 0; t < kSteps; ++t) {
          s[t][0] += __shfl_xor_sync(0xffffffffu, s[t][0], o);
          s[t][1] += __shfl_xor_sync(0xffffffffu, s[t][1], o);
        }
      float mn[2] = {mrun[0], mrun[1]};
#pragma unroll
      for (int t = 0; t < kSteps; ++t) {
        if (!ok[t]) s[t][0] = s[t][1] = -INFINITY;
        mn[0] = fmaxf(mn[0], s[t][0]);
        mn[1] = fmaxf(mn[1], s[t][1]);
      }
#pragma unroll
      for (int o = 8; o < 32; o <<= 1) {
        mn[0] = fmaxf(mn[0], __shfl_xor_sync(0xffffffffu, mn[0], o));
        mn[1] = fmaxf(mn[1], __shfl_xor_sync(0xffffffffu, mn[1], o));
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float corr = fast_exp2(mrun[h] - mn[h]);  // 0 while mrun is -inf
        float pt[kSteps];
        float l = lrun[h] * corr;
#pragma unroll
        for (int t = 0; t < kSteps; ++t) {
          pt[t] = fast_exp2(s[t][h] - mn[h]);  // 0 for masked positions
          l += pt[t];
        }
        lrun[h] = l;
        mrun[h] = mn[h];
#pragma unroll
        for (int e = 0; e < 16; ++e) oacc[h][e] *= corr;
#pragma unroll
        for (int t = 0; t < kSteps; ++t) {
          const unsigned w[8] = {va[t].x, va[t].y, va[t].z, va[t].w, vb[t].x, vb[t].y, vb[t].z, vb[t].w};
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            oacc[h][2 * k] = fmaf(pt[t], bf_lo(w[k]), oacc[h][2 * k]);
            oacc[h][2 * k + 1] = fmaf(pt[t], bf_hi(w[k]), oacc[h][2 * k + 1]);
          }
        }
      }
    };
    for (int j0 = ch.begin; j0 < ch.end; j0 += kKVTilePos) {
      const int n = min(kKVTilePos, ch.end - j0);
      const bool ok = wait_full(c, tile);
      if (ok) {
        const uint8_t *kt = slot_ptr(c, tile);
        absorb(kt, kt + kKVTileVOffset, n);
      }
      release_tile(c, tile, ok);
      ++tile;
    }
    // The new position (last split): its bf16 K/V rows were staged in smem.
    if (last) absorb(reinterpret_cast<const uint8_t *>(sU + kUKn), reinterpret_cast<const uint8_t *>(sU + kUVn), 1);

    // Groups -> warp by a reduce-scatter: afterwards lane (gq, r8) holds
    // head gq & 1, dims [base, base + 8) with base = 8 r8 + 64 (gq >> 1).
#pragma unroll
    for (int o = 8; o < 32; o <<= 1) {
      lrun[0] += __shfl_xor_sync(0xffffffffu, lrun[0], o);
      lrun[1] += __shfl_xor_sync(0xffffffffu, lrun[1], o);
    }
    const bool hb = (gq & 1) != 0, db = (gq >> 1) != 0;
    float keep[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float send = hb ? oacc[0][k] : oacc[1][k];
      keep[k] = (hb ? oacc[1][k] : oacc[0][k]) + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    float fin[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float send = db ? keep[k] : keep[8 + k];
      fin[k] = (db ? keep[8 + k] : keep[k]) + __shfl_xor_sync(0xffffffffu, send, 16);
    }
    // Cross-warp merge of the online-softmax states -> PART words.
    float *pw = sPW + warp * kPartWords;
    if (lane == 0) {
      pw[0] = mrun[0];
      pw[1] = lrun[0];
      pw[2] = mrun[1];
      pw[3] = lrun[1];
    }
    float4 *dst = reinterpret_cast<float4 *>(pw + 4 + (gq & 1) * kHeadDim + 64 * (gq >> 1) + 8 * r8);
    dst[0] = make_float4(fin[0], fin[1], fin[2], fin[3]);
    dst[1] = make_float4(fin[4], fin[5], fin[6], fin[7]);
    consumer_sync();
    // Thread i < 128: q head i / 64, dims 2 (i % 64) and 2 (i % 64) + 1.
    if (tid < kHeadDim) {
      const int hh = tid >> 6, d = 2 * (tid & 63);
      float M = -INFINITY;
#pragma unroll
      for (int q = 0; q < kConsumerWarps; ++q) M = fmaxf(M, sPW[q * kPartWords + 2 * hh]);
      float L = 0.f, O0 = 0.f, O1 = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int q = 0; q < kConsumerWarps; ++q) {
          const float mq = sPW[q * kPartWords + 2 * hh];
          if (mq != -INFINITY) {
            const float f = fast_exp2(mq - M);
            const float2 o = *reinterpret_cast<const float2 *>(sPW + q * kPartWords + 4 + hh * kHeadDim + d);
            L += sPW[q * kPartWords + 2 * hh + 1] * f;
            O0 += o.x * f;
            O1 += o.y * f;
          }
        }
      }
      {
        uint64_t *part = c.wPart + (size_t)item * kPartWords;
        put(part + 4 + hh * kHeadDim + d, ll_pack(O0, E));
        put(part + 4 + hh * kHeadDim + d + 1, ll_pack(O1, E));
        if (d == 0) {
          put(part + 2 * hh, ll_pack(M, E));
          put(part + 2 * hh + 1, ll_pack(L, E));
        }
      }
    }
    consumer_sync();  // sU scratch is reused by the next phase
    flush();
    trace_stamp(c, tid == 0, layer * 16 + 3);
  }

  // P2.5: merge the split partials of (q head h, 64 dims) -> ATT words.
  __device__ void phase_merge(unsigned E, int l) {
    const int jt = merge_task_of_cta(c.cta, c.ncta, NB);
    if (jt < 0) return;
    const int b = jt / kMergeTasks, j = jt % kMergeTasks;  // sequence, task within it
    const int h = j >> 1, half = j & 1, g = h >> 1, hl = h & 1;
    const int S = p.splits;
    const int n = S * kMergeWordsPerSplit;
    stage_list<(kMaxSplits * kMergeWordsPerSplit + kConsumerThreads - 1) / kConsumerThreads>(
        c, sU, n,
        [&](int i) -> const uint64_t * {
          const int s = i / kMergeWordsPerSplit, k = i % kMergeWordsPerSplit;
          const int word = (k < 2) ? (2 * hl + k) : (4 + hl * kHeadDim + half * kMergeDims + (k - 2));
          return c.wPart + (size_t)((b * kNumKVHeads + g) * S + s) * kPartWords + word;
        },
        E, kSitePart);
    trace_stamp(c, tid == 0, l * 16 + 4);
    if (tid < kMergeDims) {
      float M = -INFINITY;
      for (int s = 0; s < S; ++s) M = fmaxf(M, sU[s * kMergeWordsPerSplit]);
      float L = 0.f, O = 0.f;
      for (int s = 0; s < S; ++s) {
        const float ms = sU[s * kMergeWordsPerSplit];
        if (ms != -INFINITY) {
          const float f = fast_exp2(ms - M);
          L += sU[s * kMergeWordsPerSplit + 1] * f;
          O += sU[s * kMergeWordsPerSplit + 2 + tid] * f;
        }
      }
      put(c.wAtt + (NB > 1 ? (size_t)b * kWordsAtt : 0) + h * kHeadDim + half * kMergeDims + tid,
          ll_pack(O * fast_rcp(L), E));
    }
    consumer_sync();
    flush();
    trace_stamp(c, tid == 0, l * 16 + 5);
  }

  // P3: O-projection rows + residual -> A words.
  __device__ void phase_o(const LDGLayerWeights &w, unsigned E, bool stall, int l) {
    // RMSNorm weights of P4, fetched now so that their latency is hidden.
    nw_pref = load_norm_pairs((const __nv_bfloat16 *)w.post_attn_layernorm_weight, tid);
    const Range R = o_rows(c.cta, c.ncta);
    const bool tiles = wait_tiles(tiles_of(R, kOTileRows));
    // Test hook: 0xFFFFFFFF is never an epoch, so this wait can only expire.
    stage_vec<kQSize, kStageCopy>(c, sAtt, nullptr, c.wAtt, stall ? 0xFFFFFFFFu : E, kSiteAtt, nullptr, NormPairs{});
    trace_stamp(c, tid == 0, l * 16 + 6);
    fma_ksplit_phase<2, kOutO>(tiles, sAtt, R.begin, R.end, kOTileRows, kQSize * 2, E);
    flush();
    trace_stamp(c, tid == 0, l * 16 + 7);
  }

  // P4: RMSNorm(a) then gate/up rows, SiLU(gate) * up -> M words.
  __device__ void phase_gate_up(const LDGLayerWeights &w, unsigned E, int l) {
    const NormPairs nw = nw_pref;  // fetched in P3
    const Range R = gu_rows(c.cta, c.ncta);
    const bool tiles = wait_tiles(tiles_of(R, kGUTileRows));
    const float ss = stage_vec<kHidden, kStageNorm>(c, sA, reinterpret_cast<uint8_t *>(sXW), c.wA, E, kSiteA, red_a, nw);
    trace_stamp(c, tid == 0, l * 16 + 8);
    fma_rows_phase<kOutGU, 3>(tiles, sXW, R.begin, R.end, kGUTileRows, 4096, rsqrtf(ss / (float)kHidden + kRmsEps), E);
    flush();
    trace_stamp(c, tid == 0, l * 16 + 9);
  }

  // P5: down rows + residual -> X words (next layer's input).
  __device__ void phase_down(const LDGLayerWeights &w, unsigned E, int l) {
    // RMSNorm weights of the next P1 (or of the final norm), fetched now.
    nw_pref = load_norm_pairs(
        (l + 1 < p.num_layers) ? (const __nv_bfloat16 *)p.layers[l + 1].input_layernorm_weight : p.final_norm, tid);
    const Range R = d_rows(c.cta, c.ncta);
    const bool tiles = wait_tiles(tiles_of(R, kDTileRows));
    stage_vec<kInter, kStageCopy>(c, sU, nullptr, c.wM, E, kSiteM, nullptr, NormPairs{});
    trace_stamp(c, tid == 0, l * 16 + 10);
    fma_ksplit_phase<3, kOutDown>(tiles, sU, R.begin, R.end, kDTileRows, kDRowPitch, E);
    flush();
    trace_stamp(c, tid == 0, l * 16 + 11);
  }

  // k-th largest (1 <= k <= n) of the n keys get(0 .. n-1), all consumer
  // threads: most-significant-digit radix select, 4 passes of 8 bits with a
  // 256-bin histogram in smem (hist) and the pass result in bc[0..1].
  template <class GetKey>
  __device__ unsigned kth_largest_key(int n, int k, GetKey get, unsigned *hist, unsigned *bc) {
    unsigned prefix = 0u, mask = 0u;
    unsigned kk = (unsigned)k;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = tid; i < 256; i += kConsumerThreads) hist[i] = 0u;
      consumer_sync();
      for (int i = tid; i < n; i += kConsumerThreads) {
        const unsigned key = get(i);
        if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
      }
      consumer_sync();
      if (warp == 0) {
        // lane l sums bins 255 - 8l .. 248 - 8l (descending digits)
        unsigned cnt[8], sum = 0u;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          cnt[j] = hist[255 - 8 * lane - j];
          sum += cnt[j];
        }
        unsigned incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const unsigned t = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += t;
        }
        const unsigned excl = incl - sum;
        if (excl < kk && kk <= incl) {
          unsigned run = excl;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (run < kk && kk <= run + cnt[j]) {
              bc[0] = 255u - 8u * lane - j;
              bc[1] = kk - run;
            }
            run += cnt[j];
          }
        }
      }
      consumer_sync();
      prefix |= bc[0] << shift;
      mask |= 255u << shift;
      kk = bc[1];
    }
    return prefix;
  }

  // Top-k sampling: every CTA publishes the keys of its top_k logits, every
  // CTA then finds the global top_k-th key tau from all candidates and draws
  // its local Gumbel-max among its logits with key >= tau; the usual argmax
  // exchange picks the grid's winner (an exact draw from softmax(logits / T)
  // restricted to the logits >= the top_k-th largest).
  __device__ void topk_select(unsigned E) {
    const Range R = lm_rows(c.cta, c.ncta);
    const int n = R.end - R.begin, k = p.top_k;
    unsigned *hist = reinterpret_cast<unsigned *>(sA);  // free during the LM head
    unsigned *bc = hist + 256;
    const float *vals = sU + kHidden;  // this CTA's logits, written by the LM-head emit
    consumer_sync();  // every row's logit is in smem
    const unsigned kc = kth_largest_key(n, k, [&](int i) { return float_order_key(vals[i]); }, hist, bc);
    if (tid == 0) bc[2] = 0u;
    consumer_sync();
    uint64_t *mine = c.wTopk + (size_t)c.cta * k;
    for (int i = tid; i < n; i += kConsumerThreads) {
      const unsigned key = float_order_key(vals[i]);
      if (key > kc && live()) put(mine + atomicAdd(&bc[2], 1u), ll_pack_u(key, E));
    }
    consumer_sync();
    for (int i = (int)bc[2] + tid; i < k; i += kConsumerThreads)
      if (live()) put(mine + i, ll_pack_u(kc, E));
    flush();
    // wait for every CTA's candidates (word j * kConsumerThreads + tid of
    // this thread, at most 64 per thread)
    const int total = c.ncta * k;
    unsigned long long pending = 0ull;
    for (int j = 0; j < 64 && j * kConsumerThreads + tid < total; ++j) pending |= 1ull << j;
    if (*c.abort_flag) pending = 0ull;
    Waiter w;
    while (pending) {
      for (int j = 0; j < 64; ++j) {
        if ((pending >> j) & 1ull) {
          if (ll_flag(ll_load(c.wTopk + j * kConsumerThreads + tid)) == E) pending &= ~(1ull << j);
        }
      }
      if (!pending || !w.keep_going(c, kSiteTopk)) break;
    }
    consumer_sync();
    const unsigned tau = kth_largest_key(
        total, k, [&](int i) { return (unsigned)(ll_load(c.wTopk + i) & 0xffffffffull); }, hist, bc);
    lm_best = -INFINITY;
    lm_best_i = 0x7fffffff;
    for (int i = tid; i < n; i += kConsumerThreads) {
      const float v = vals[i];
      if (float_order_key(v) >= tau) {
        const int row = R.begin + i;
        const float key = (p.inv_temp > 0.f) ? fmaf(v, p.inv_temp, gumbel_noise(p.seed, lm_pos, row)) : v;
        if (key > lm_best || (key == lm_best && row < lm_best_i)) {
          lm_best = key;
          lm_best_i = row;
        }
      }
    }
  }

  // Final RMSNorm + LM head rows + CTA argmax -> ARG words.
  __device__ void phase_lm_head(int step, unsigned E_x, unsigned E) {
    const NormPairs nw = nw_pref;  // fetched in the last P5
    uint8_t *bop = reinterpret_cast<uint8_t *>(sU);
    const Range R = lm_rows(c.cta, c.ncta);
    tc_prewait(R.begin, R.end, kLMTileRows);
    const float ss = stage_vec<kHidden, kStageNormFrag>(c, sX, bop, c.wX, E_x, kSiteX, red_lm, nw);
    trace_stamp(c, tid == 0, p.num_layers * 16 + 0);
    const float rstd = rsqrtf(ss / (float)kHidden + kRmsEps);
    if (p.final_hidden && c.cta == 0 && step == p.num_steps - 1 && live()) {
      for (int i = tid; i < kHidden; i += kConsumerThreads)
        p.final_hidden[i] = (sX[i] * rstd) * __bfloat162float(p.final_norm[i]);
    }
    lm_best = -INFINITY;
    lm_best_i = 0x7fffffff;
    lm_logits = p.logits ? (p.logits + (size_t)step * kVocab) : nullptr;
    lm_pos = p.start_pos + step;
    const TcJob job{kTcRow, kOutLM, R.begin, R.end, kLMTileRows, rstd, E};
    tc_phase(job, bop);
    if constexpr (kFeat) {
      if (p.top_k > 0) topk_select(E);
    }
    float best = lm_best;
    int best_i = lm_best_i;
    // warp argmax (largest value, lowest row on ties)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
      if (ov > best || (ov == best && oi < best_i)) {
        best = ov;
        best_i = oi;
      }
    }
    if (lane == 0) {
      c.warp_best_v[warp] = best;
      c.warp_best_i[warp] = best_i;
    }
    consumer_sync();
    if (tid == 0) {
      unsigned bk = 0;
      int bi = 0x7fffffff;
      for (int q = 0; q < kConsumerWarps; ++q) {
        const float v = c.warp_best_v[q];
        const int i = c.warp_best_i[q];
        if (i == 0x7fffffff) continue;
        const unsigned k = float_order_key(v);
        if (arg_better(k, i, bk, bi)) {
          bk = k;
          bi = i;
        }
      }
      if (bi == 0x7fffffff) bi = R.begin;  // CTA without rows (not on B200)
      put(c.wArg + 2 * c.cta, ll_pack_u(bk, E));
      put(c.wArg + 2 * c.cta + 1, ll_pack_u((unsigned)bi, E));
    }
    flush();
    consumer_sync();
    publish_kv(step);
    trace_stamp(c, tid == 0, p.num_layers * 16 + 1);
  }

  // Publish this step's K/V rows for the next step's TMA reads, after the
  // ARG words (off the step's critical path): one gpu-scope fence orders
  // every row written since (the CTA synchronized with their writers at the
  // named barriers in between), then the flags as relaxed stores.
  __device__ void publish_kv(int step) {
    if (kv_written && tid == 0 && live()) {
      __threadfence();
      const int item = item_of_cta(c.cta, p.splits, NB);
      const int g = (item / p.splits) % kNumKVHeads;
      const int b = (NB > 1) ? item / (kNumKVHeads * p.splits) : 0;
      for (int l = 0; l < p.num_layers; ++l)
        if (kv_written & (1ull << l))
          st_relaxed_u32(&c.ctrl->kv_ready[(b * kMaxLayers + l) * kNumKVHeads + g], epoch_of(c, step, l, p.num_layers));
    }
    kv_written = 0;
  }

  // Token consumed by step t.
  __device__ int step_token(int t) {
    int tok;
    if (t < p.n_forced) {
      tok = __ldg(p.forced + t);
    } else if (t == 0) {
      tok = p.first_token;
    } else {
      tok = read_argmax(c, epoch_of(c, t - 1, p.num_layers, p.num_layers));
    }
    if (tok < 0 || tok >= kVocab) {
      if (tid == 0) raise_error(c, QMK_ERR_TOKEN, kSiteToken);
      tok = 0;
    }
    return tok;
  }

  int steps_run = 0;  // steps executed (num_steps unless stopped at EOS)

  __device__ void run() {
    if constexpr (NB > 1) {
      run_nb();
      return;
    }
    const int L = p.num_layers;
    steps_run = p.num_steps;
    for (int t = 0; t < p.num_steps; ++t) {
      c.trace = (kFeat && p.trace && t == p.trace_step) ? p.trace + (size_t)c.cta * kTraceStride : nullptr;
      c.trace_tile0 = tile;
      trace_stamp(c, tid == 0, L * 16 + 5);
      // CTA 0 records the previous step's argmax (needed even when forced).
      if (t > 0 && c.cta == 0) {
        const int prev = read_argmax(c, epoch_of(c, t - 1, L, L));
        if (tid == 0 && live() && p.out_log) p.out_log[t - 1] = prev;
      }
      nw_pref = load_norm_pairs((const __nv_bfloat16 *)p.layers[0].input_layernorm_weight, tid);
      const int tok = step_token(t);
      // EOS stop: the token step t would consume was generated (not forced)
      // and is the end-of-sequence id.  Every consumer thread read the same
      // token, so all leave here; the producer warp sees the stop step and
      // stops issuing (it drains what it issued for this step).
      if (p.eos_token >= 0 && t > 0 && t >= p.n_forced && tok == p.eos_token) {
        steps_run = t;
        if (tid == 0) *c.stop_step = t;
        break;
      }
      // Layer-0 input: the embedding row (bf16 -> fp32) and its sum of squares.
      float x_ss;
      {
        const __nv_bfloat16 *erow = p.embed + (size_t)tok * kHidden;
        float ss = 0.f;
        for (int i = tid; i < kHidden / 4; i += kConsumerThreads) {
          const uint2 v = __ldg(reinterpret_cast<const uint2 *>(erow) + i);
          const float e0 = bf_lo(v.x), e1 = bf_hi(v.x), e2 = bf_lo(v.y), e3 = bf_hi(v.y);
          sX[4 * i + 0] = e0;
          sX[4 * i + 1] = e1;
          sX[4 * i + 2] = e2;
          sX[4 * i + 3] = e3;
          ss += e0 * e0 + e1 * e1 + e2 * e2 + e3 * e3;
        }
        ss = warp_sum(ss);
        if (lane == 0) red_e[warp] = ss;
        consumer_sync();
        x_ss = 0.f;
#pragma unroll
        for (int q = 0; q < kConsumerWarps; ++q) x_ss += red_e[q];
      }
      for (int l = 0; l < L; ++l) {
        c.cur_layer = l;
        const LDGLayerWeights w = p.layers[l];
        const unsigned E = epoch_of(c, t, l, L);
        phase_qkv(w, E, l, l > 0 ? epoch_of(c, t, l - 1, L) : 0u, x_ss);
        phase_attention(w, l, t, E);
        phase_merge(E, l);
        phase_o(w, E, p.debug_stall == c.cta + 1 && t == 0 && l == 0, l);
        phase_gate_up(w, E, l);
        phase_down(w, E, l);
      }
      phase_lm_head(t, epoch_of(c, t, L - 1, L), epoch_of(c, t, L, L));
    }
    if (c.cta == 0) {
      // After an EOS stop the last step's token (the EOS) is already in the log.
      const int last = (steps_run == p.num_steps) ? read_argmax(c, epoch_of(c, p.num_steps - 1, L, L)) : p.eos_token;
      if (tid == 0 && live()) {
        if (p.out_log && steps_run == p.num_steps) p.out_log[p.num_steps - 1] = last;
        if (p.out_token) *p.out_token = last;
        if (p.steps_done) *p.steps_done = steps_run;
      }
      if (tid == 0 && !live() && p.out_token) *p.out_token = -1;
    }
  }

  // ---------------------------------------------------- batched instance
  // NB > 1 sequences decoded together (greedy).  A GEMV phase stages the
  // inputs of all NB sequences at once (one poll loop, one barrier) and
  // makes ONE pass over its ring tiles in which every weight meets all NB
  // inputs, so every weight byte is read from HBM once per step for all
  // sequences: q|k|v, gate/up and the LM head (K = 1024, many rows) on the
  // tensor cores with the NB inputs as the N = 16 NB columns of the B
  // operand (tc_phase_nb); O and down (a few rows, K = 2048 / 3072) as a
  // K-split on the CUDA cores (fma_ksplit_nb).  Attention items and merge
  // tasks are per (sequence, ...).

  // Layer-0 input: the embedding row of `tok` into dst; returns its sum of
  // squares (one consumer barrier, reduction slots `red`).
  __device__ float embed_row(int tok, float *dst, float *red) {
    const __nv_bfloat16 *erow = p.embed + (size_t)tok * kHidden;
    float ss = 0.f;
    for (int i = tid; i < kHidden / 4; i += kConsumerThreads) {
      const uint2 v = __ldg(reinterpret_cast<const uint2 *>(erow) + i);
      const float e0 = bf_lo(v.x), e1 = bf_hi(v.x), e2 = bf_lo(v.y), e3 = bf_hi(v.y);
      dst[4 * i + 0] = e0;
      dst[4 * i + 1] = e1;
      dst[4 * i + 2] = e2;
      dst[4 * i + 3] = e3;
      ss += e0 * e0 + e1 * e1 + e2 * e2 + e3 * e3;
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    consumer_sync();
    float total = 0.f;
#pragma unroll
    for (int q = 0; q < kConsumerWarps; ++q) total += red[q];
    return total;
  }

  // Inputs of a normalized row phase for all NB sequences, staged side by
  // side: raw x_b at sX + b * kHidden (the X, A and ATT regions, 16 KB) and
  // the B operand of the x_b * w in the U and x*w regions (16 KB).
  static_assert(kSmA == kSmX + 4 * kHidden && kSmAtt == kSmA + 4 * kHidden && kSmU == kSmAtt + 4 * kQSize &&
                    kSmXW == kSmU + 4 * kInter,
                "activation regions are contiguous");
  static_assert(NB * kHidden <= 2 * kHidden + kQSize && NB * kHidden <= kInter + kHidden, "staged inputs fit");

  // K-split GEMV of NV staged inputs (x_j at xin + j * K, K = 1024 KC;
  // sequences b0 .. b0 + NV - 1) in one pass: the 128-element blocks of K go
  // round-robin to the warps, every warp multiplies its blocks of every row
  // with the NV inputs (each weight read once), per row a transposing
  // butterfly leaves input j's partial in lane 8j, the partials of all rows
  // and inputs meet in shared memory (`part`) behind one barrier, and thread
  // (row, j) adds its row's partials in warp order and emits.  Rows per CTA
  // <= kKsplitGroupRows.
  template <int KC, int OUT, int NV>
  __device__ void fma_ksplit_nb(bool ok, const float *xin, int b0, float *part, int r0, int r1, int tile_rows,
                                int pitch, unsigned E) {
    static_assert(NV >= 1 && NV <= 4, "one lane group of 8 per input");
    constexpr int K = 1024 * KC;
    constexpr int kBlocks = 8 * KC;
    constexpr int kMine = (kBlocks + kConsumerWarps - 1) / kConsumerWarps;
    constexpr int RB = kKsplitRows;
    constexpr int RG = kKsplitGroupRows;
    const TcJob job{kTcRow, OUT, r0, r1, tile_rows, 1.f, E};
    const int n = r1 - r0;  // <= RG (checked on the host)
    float4 xv[kMine][NV];
#pragma unroll
    for (int q = 0; q < kMine; ++q) {
      const int blk = warp + kConsumerWarps * q;
#pragma unroll
      for (int b = 0; b < NV; ++b)
        xv[q][b] = (blk < kBlocks) ? reinterpret_cast<const float4 *>(xin + b * K)[lane + 32 * blk]
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int i0 = 0; i0 < n; i0 += RB) {
      float acc[RB][NV][2];
#pragma unroll
      for (int r = 0; r < RB; ++r)
#pragma unroll
        for (int b = 0; b < NV; ++b) acc[r][b][0] = acc[r][b][1] = 0.f;
      if (ok) {
#pragma unroll
        for (int r = 0; r < RB; ++r) {
          if (i0 + r < n) {
            const uint8_t *rp = row_ptr(i0 + r, tile_rows, pitch, 8 * lane);
#pragma unroll
            for (int q = 0; q < kMine; ++q) {
              const int blk = warp + kConsumerWarps * q;
              if (blk < kBlocks) {
                const uint2 wv = *reinterpret_cast<const uint2 *>(rp + 256 * blk);
#pragma unroll
                for (int b = 0; b < NV; ++b) dot4(acc[r][b][0], acc[r][b][1], wv, xv[q][b]);
              }
            }
          }
        }
      }
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        float v[4];
#pragma unroll
        for (int b = 0; b < 4; ++b) v[b] = (b < NV) ? acc[r][b < NV ? b : 0][0] + acc[r][b < NV ? b : 0][1] : 0.f;
        const float wsum = reduce4_transpose(v);  // lane 8j: input j
        if ((lane & 7) == 0 && (lane >> 3) < NV && i0 + r < n) part[(warp * RG + i0 + r) * NV + (lane >> 3)] = wsum;
      }
    }
    consumer_sync();
    if (ok && tid < n * NV) {
      const int i = tid / NV, b = tid % NV;
      float sum = 0.f;
#pragma unroll
      for (int q = 0; q < kConsumerWarps; ++q) sum += part[(q * RG + i) * NV + b];
      cur_b = b0 + b;
      tc_emit(job, r0 + i, sum, 0.f);
    }
  }

  __device__ void phase_qkv_nb(unsigned E, unsigned x_flag, const int (&toks)[NB], const __nv_bfloat16 *nw_ptr) {
    const NormPairs nw = nw_pref;
    const Range R = qkv_rows(c.cta, c.ncta), Ro = o_rows(c.cta, c.ncta);
    uint8_t *bop = reinterpret_cast<uint8_t *>(sU);  // the NB inputs x_b * w (16 KB)
    tc_prewait(R.begin, R.end, kQKVTileRows);
    float rstd[NB];
    if (x_flag) {
      float ss[NB];
      stage_vecs<kHidden, NB, kStageNormFrag>(c, sX, sU, c.wX, kWordsX, x_flag, kSiteX, red_x, nw_ptr, ss);
#pragma unroll
      for (int b = 0; b < NB; ++b) rstd[b] = rsqrtf(ss[b] / (float)kHidden + kRmsEps);
    } else {
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        // back-to-back embeddings alternate their reduction slots
        const float ss = embed_row(toks[b], sX + b * kHidden, (b & 1) ? red_e : red_x);
        build_norm_bop_slot<NB>(bop, b, sX + b * kHidden, nw, tid);
        rstd[b] = rsqrtf(ss / (float)kHidden + kRmsEps);
      }
      fence_proxy_async_smem();
      consumer_sync();  // the B operand of the embeddings
    }
    const int no = Ro.end - Ro.begin;
    if (tid < NB * no) sResO[(tid / no) * kMaxResRows + tid % no] = sX[(tid / no) * kHidden + Ro.begin + tid % no];
    const TcJob job{kTcRow, kOutQKV, R.begin, R.end, kQKVTileRows, 1.f, E};
    tc_phase_nb(job, bop, rstd);
    consumer_sync();  // the next phase writes its scratch over the staged inputs
  }

  __device__ void phase_o_nb(const LDGLayerWeights &w, unsigned E) {
    nw_pref = load_norm_pairs((const __nv_bfloat16 *)w.post_attn_layernorm_weight, tid);
    const Range R = o_rows(c.cta, c.ncta);
    const int ntiles = tiles_of(R, kOTileRows);
    const bool tiles = wait_tiles(ntiles);
    // the NB attention outputs side by side over all activation regions (32 KB)
    static_assert(NB * kQSize * 4 == kSmMisc - kSmX, "attention outputs fill the activation regions");
    float unused[NB];
    stage_vecs<kQSize, NB, kStageCopy>(c, sX, nullptr, c.wAtt, kWordsAtt, E, kSiteAtt, nullptr, nullptr, unused);
    static_assert(kConsumerWarps * kKsplitGroupRows * NB <= 2 * 16 * kKsplitGroupRows, "partials fit");
    fma_ksplit_nb<2, kOutO, NB>(tiles, sX, 0, sPart, R.begin, R.end, kOTileRows, kQSize * 2, E);
    release_tiles(ntiles, tiles);
  }

  __device__ void phase_gu_nb(unsigned E, const __nv_bfloat16 *nw_ptr) {
    const Range R = gu_rows(c.cta, c.ncta), Rd = d_rows(c.cta, c.ncta);
    uint8_t *bop = reinterpret_cast<uint8_t *>(sU);
    tc_prewait(R.begin, R.end, kGUTileRows);
    float ss[NB], rstd[NB];
    stage_vecs<kHidden, NB, kStageNormFrag>(c, sX, sU, c.wA, kWordsA, E, kSiteA, red_x, nw_ptr, ss);
#pragma unroll
    for (int b = 0; b < NB; ++b) rstd[b] = rsqrtf(ss[b] / (float)kHidden + kRmsEps);
    const int nd = Rd.end - Rd.begin;
    if (tid < NB * nd) sResD[(tid / nd) * kMaxResRows + tid % nd] = sX[(tid / nd) * kHidden + Rd.begin + tid % nd];
    const TcJob job{kTcGU, kOutGU, R.begin, R.end, kGUTileRows, 1.f, E};
    tc_phase_nb(job, bop, rstd);
    consumer_sync();  // the next phase stages over the inputs
  }

  __device__ void phase_down_nb(unsigned E, int l) {
    nw_pref = load_norm_pairs(
        (l + 1 < p.num_layers) ? (const __nv_bfloat16 *)p.layers[l + 1].input_layernorm_weight : p.final_norm, tid);
    const Range R = d_rows(c.cta, c.ncta);
    const int ntiles = tiles_of(R, kDTileRows);
    const bool tiles = wait_tiles(ntiles);
    // two sequences per pass: their MLP inputs (2 x 12 KB) in the activation
    // regions, the partials of the two passes in separate halves of the slots
    constexpr int kPer = 2;
    static_assert(NB % kPer == 0 && kPer * kInter * 4 <= kSmMisc - kSmX, "MLP inputs fit");
    static_assert(2 * kConsumerWarps * kKsplitGroupRows * kPer <= 2 * 16 * kKsplitGroupRows, "partials fit");
#pragma unroll 1
    for (int b0 = 0; b0 < NB; b0 += kPer) {
      float unused[kPer];
      stage_vecs<kInter, kPer, kStageCopy>(c, sX, nullptr, c.wM + (size_t)b0 * kWordsM, kWordsM, E, kSiteM, nullptr,
                                           nullptr, unused);
      fma_ksplit_nb<3, kOutDown, kPer>(tiles, sX, b0, sPart + (b0 / kPer & 1) * (kConsumerWarps * kKsplitGroupRows * kPer),
                                       R.begin, R.end, kDTileRows, kDRowPitch, E);
    }
    release_tiles(ntiles, tiles);
  }

  // LM head of all NB sequences in one pass over this CTA's vocabulary rows
  // on the tensor cores (tc_phase_nb, the NB final-normed inputs as one B
  // operand, N = 16 NB): the weights cross HBM once per step for all
  // sequences.  Reader lane q of a segment keeps the running argmax of
  // sequence q >> 1 over the rows it emits; per sequence, a butterfly over
  // the segments of a warp and a pass over the warps in warp order give the
  // CTA's candidate (largest logit, lowest row on ties).
  __device__ void phase_lm_nb(int step, unsigned E_x, unsigned E) {
    static_assert(NB == 4, "one sequence per lane pair of a segment");
    const Range R = lm_rows(c.cta, c.ncta);
    uint8_t *bop = reinterpret_cast<uint8_t *>(sU);
    tc_prewait(R.begin, R.end, kLMTileRows);
    float ss[NB], rstd[NB];
    stage_vecs<kHidden, NB, kStageNormFrag>(c, sX, sU, c.wX, kWordsX, E_x, kSiteX, red_x, p.final_norm, ss);
#pragma unroll
    for (int b = 0; b < NB; ++b) rstd[b] = rsqrtf(ss[b] / (float)kHidden + kRmsEps);
    lm_best = -INFINITY;
    lm_best_i = 0x7fffffff;
    const TcJob job{kTcRow, kOutLM, R.begin, R.end, kLMTileRows, 1.f, E};
    tc_phase_nb(job, bop, rstd);
    float best = lm_best;
    int best_i = lm_best_i;
#pragma unroll
    for (int o = 8; o < 32; o <<= 1) {  // the warp's segments, same q
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
      if (ov > best || (ov == best && oi < best_i)) {
        best = ov;
        best_i = oi;
      }
    }
    float *bv = sPart;  // [kConsumerWarps][NB] (the K-split partials are free here)
    int *bi = reinterpret_cast<int *>(sPart + 64);
    static_assert(kConsumerWarps * NB <= 64, "argmax slots");
    if (lane < 8 && (lane & 1) == 0) {  // issuer warps: no rows (sentinel index)
      bv[warp * NB + (lane >> 1)] = best;
      bi[warp * NB + (lane >> 1)] = best_i;
    }
    consumer_sync();
    if (tid < NB) {
      unsigned bk = 0;
      int bidx = 0x7fffffff;
      for (int q = 0; q < kConsumerWarps; ++q) {
        const int i = bi[q * NB + tid];
        if (i == 0x7fffffff) continue;
        const unsigned k = float_order_key(bv[q * NB + tid]);
        if (arg_better(k, i, bk, bidx)) {
          bk = k;
          bidx = i;
        }
      }
      if (bidx == 0x7fffffff) bidx = R.begin;
      uint64_t *arg = c.wArg + (size_t)tid * kWordsArg;
      put(arg + 2 * c.cta, ll_pack_u(bk, E));
      put(arg + 2 * c.cta + 1, ll_pack_u((unsigned)bidx, E));
    }
    consumer_sync();  // the argmax slots and the inputs are reused next step
    publish_kv(step);
  }

  __device__ void run_nb() {
    const int L = p.num_layers;
    steps_run = p.num_steps;
    int toks[NB];
    for (int t = 0; t < p.num_steps; ++t) {
      c.trace_tile0 = tile;
      nw_pref = load_norm_pairs((const __nv_bfloat16 *)p.layers[0].input_layernorm_weight, tid);
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        int tok = (t == 0) ? __ldg(p.first_tokens_b + b) : read_argmax(c, epoch_of(c, t - 1, L, L), b);
        if (tok < 0 || tok >= kVocab) {
          if (tid == 0) raise_error(c, QMK_ERR_TOKEN, kSiteToken);
          tok = 0;
        }
        toks[b] = tok;
      }
      // CTA 0 records the previous step's tokens
      if (t > 0 && c.cta == 0 && tid == 0 && p.out_log) {
#pragma unroll
        for (int b = 0; b < NB; ++b) p.out_log[(size_t)(t - 1) * NB + b] = toks[b];
      }
      for (int l = 0; l < L; ++l) {
        c.cur_layer = l;
        const LDGLayerWeights w = p.layers[l];
        const unsigned E = epoch_of(c, t, l, L);
        phase_qkv_nb(E, l > 0 ? epoch_of(c, t, l - 1, L) : 0u, toks,
                     (const __nv_bfloat16 *)w.input_layernorm_weight);
        phase_attention(w, l, t, E);
        phase_merge(E, l);
        phase_o_nb(w, E);
        phase_gu_nb(E, (const __nv_bfloat16 *)w.post_attn_layernorm_weight);
        phase_down_nb(E, l);
      }
      phase_lm_nb(t, epoch_of(c, t, L - 1, L), epoch_of(c, t, L, L));
    }
    if (c.cta == 0) {
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const int last = read_argmax(c, epoch_of(c, p.num_steps - 1, L, L), b);
        if (tid == 0 && p.out_log) p.out_log[(size_t)(p.num_steps - 1) * NB + b] = last;
      }
    }
  }
};

template <bool kFeat, int NB = 1>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ int s_abort;
  __shared__ int s_stop;
  __shared__ unsigned s_epoch;
  Ctx c;
  c.ring = smem + kSmRing;
  c.full = reinterpret_cast<uint64_t *>(smem + kSmMisc);
  c.empty = c.full + kNumSlots;
  c.warp_best_v = reinterpret_cast<float *>(smem + kSmMisc + kMiscBestV);
  c.warp_best_i = reinterpret_cast<int *>(smem + kSmMisc + kMiscBestI);
  c.abort_flag = &s_abort;
  c.stop_step = &s_stop;
  c.ctrl = reinterpret_cast<Ctrl *>(p.ws);
  c.wX = reinterpret_cast<uint64_t *>(p.ws + kOffX);
  c.wQKV = reinterpret_cast<uint64_t *>(p.ws + kOffQKV);
  c.wPart = reinterpret_cast<uint64_t *>(p.ws + kOffPart);
  c.wAtt = reinterpret_cast<uint64_t *>(p.ws + kOffAtt);
  c.wA = reinterpret_cast<uint64_t *>(p.ws + kOffA);
  c.wM = reinterpret_cast<uint64_t *>(p.ws + kOffM);
  c.wArg = reinterpret_cast<uint64_t *>(p.ws + kOffArg);
  c.wTopk = reinterpret_cast<uint64_t *>(p.ws + kOffTopk);
  c.cta = blockIdx.x;
  c.ncta = gridDim.x;
  c.timeout_ns = p.timeout_ns;
  c.cur_layer = 0;
  c.trace = nullptr;
  c.trace_tile0 = 0;
  c.poll_backoff_ns = kFeat ? p.poll_backoff_ns : 0u;
  c.tuning = kFeat ? p.tuning : 0u;
  c.mma_bar = reinterpret_cast<uint64_t *>(smem + kSmMisc + kMiscMmaBar);
  c.tmem_free = reinterpret_cast<uint64_t *>(smem + kSmMisc + kMiscTmemFree);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kSmMisc + kMiscTmem);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kNumSlots; ++s) {
      mbar_init(&c.full[s], 1);
      mbar_init(&c.empty[s], kConsumerWarps);
    }
    for (int b = 0; b < kTmemBufs; ++b) {
      mbar_init(&c.mma_bar[b], 1);
      mbar_init(&c.tmem_free[b], 4);
    }
    fence_mbar_init();
    s_abort = 0;
    s_stop = 0x7fffffff;
    s_epoch = ld_relaxed_u32(&c.ctrl->epoch);
    // The tensor-core operands use 1 KB swizzle atoms: refuse to run on a
    // misaligned dynamic shared memory window instead of computing garbage.
    if (smem_addr(smem) & 1023u) raise_error_at(&s_abort, c.ctrl, QMK_ERR_SMEM, 0u, c.cta, 0);
  }
  // One CTA per SM: the TMEM allocation (warp 0) never has to wait.
  if (threadIdx.x < 32) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  c.E0 = s_epoch;
  c.tmem = *tmem_slot;

  if (threadIdx.x >= kConsumerThreads) {
    if ((threadIdx.x & 31) == 0) {
      Producer<kFeat, NB> prod(c, p);
      prod.run();
    }
  } else {
    Consumer<kFeat, NB> cons(c, p, smem);
    cons.run();
    cons.drain_mma();
  }
  tc_fence_before_sync();
  __syncthreads();
  if (threadIdx.x < 32) {
    tc_fence_after_sync();
    tmem_dealloc(c.tmem, kTmemCols);
  }

  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned done = atomicAdd(&c.ctrl->exit_count, 1u);
    if (done == (unsigned)c.ncta - 1u) {
      __threadfence();
      const unsigned used = (unsigned)p.num_steps * (unsigned)(p.num_layers + 1) + 1u;
      unsigned next = c.E0 + used;
      if (next > kEpochWrap) {
        // Epochs restart from 1.  Dataflow words are written with atomic max
        // on the epoch, so the old high-epoch words must be cleared first;
        // every other CTA has finished, nothing reads them concurrently.
        next = 0;
        uint64_t *ll = reinterpret_cast<uint64_t *>(p.ws + kOffX);
        const long long nwords = (kOffLLEnd - kOffX) / 8;
        for (long long i = 0; i < nwords; ++i) ll[i] = 0ull;
        __threadfence();
      }
      const unsigned code = ld_relaxed_u32(&c.ctrl->err_code);
      const unsigned info = ld_relaxed_u32(&c.ctrl->err_info);
      const unsigned launches = c.ctrl->launches + 1u;
      c.ctrl->epoch = next;
      c.ctrl->err_code = 0;
      c.ctrl->err_info = 0;
      c.ctrl->launches = launches;
      c.ctrl->exit_count = 0;
      if (p.status) {
        volatile QmkStatus *st = p.status;
        st->error_code = code;
        st->error_info = info;
        st->epoch = next;
        st->launches = launches;
        __threadfence_system();
      }
    }
  }
}

}  // namespace qmk

// =============================================================================
// Host side: C ABI
// =============================================================================

namespace {

thread_local int g_last_error = QMK_OK;
thread_local char g_last_msg[512] = "";

int set_error(int code, const char *fmt, ...) {
  g_last_error = code;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_msg, sizeof(g_last_msg), fmt, ap);
  va_end(ap);
  return code;
}

int clear_error() {
  g_last_error = QMK_OK;
  g_last_msg[0] = '\0';
  return QMK_OK;
}

}  // namespace

// Error reporting shared with the library's other translation units (not
// part of the exported C ABI).
__attribute__((visibility("hidden"))) int qmk_internal_set_error(int code, const char *msg) {
  return set_error(code, "%s", msg);
}
__attribute__((visibility("hidden"))) int qmk_internal_clear_error() { return clear_error(); }

namespace {

struct DeviceState {
  bool attr_set = false;
  int num_sms = 0;
  void *default_ws = nullptr;
  QmkStatus *default_status_host = nullptr;
  QmkStatus *default_status_dev = nullptr;
};

constexpr int kMaxDevices = 64;
DeviceState g_devices[kMaxDevices];
std::mutex g_mutex;

int current_device(int *dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return set_error(QMK_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (*dev < 0 || *dev >= kMaxDevices) return set_error(QMK_ERR_CUDA, "device %d out of range", *dev);
  return QMK_OK;
}

// Kernel attributes + SM count for the current device (once per device).
int prepare_device(int dev) {
  DeviceState &ds = g_devices[dev];
  if (ds.attr_set) return QMK_OK;
  cudaError_t e = cudaFuncSetAttribute(qmk::decode_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       qmk::kSmBytes - 0);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(qmk::decode_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, qmk::kSmBytes);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(qmk::decode_kernel<false, qmk::kBatchSeqs>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             qmk::kSmBytes);
  if (e != cudaSuccess)
    return set_error(QMK_ERR_CUDA, "cudaFuncSetAttribute(max dynamic smem %d): %s", qmk::kSmBytes,
                     cudaGetErrorString(e));
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return set_error(QMK_ERR_CUDA, "SM count: %s", cudaGetErrorString(e));
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qmk::decode_kernel<false>, qmk::kThreads,
                                                    qmk::kSmBytes);
  if (e == cudaSuccess && per_sm >= 1) {
    int per_sm_topk = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm_topk, qmk::decode_kernel<true>, qmk::kThreads,
                                                      qmk::kSmBytes);
    if (per_sm_topk < per_sm) per_sm = per_sm_topk;
  }
  if (e != cudaSuccess) return set_error(QMK_ERR_CUDA, "occupancy query: %s", cudaGetErrorString(e));
  if (per_sm < 1) return set_error(QMK_ERR_LAUNCH, "decode kernel does not fit on one SM");
  ds.num_sms = sms;
  ds.attr_set = true;
  return QMK_OK;
}

bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace

extern "C" {

size_t qmk_workspace_bytes(void) { return (size_t)qmk::kWorkspaceBytes; }

const char *qmk_version(void) { return "qwen_megakernel_b200 0.1 (sm_100a)"; }

int qmk_trace_words(void) { return qmk::kTraceStride; }

const char *qmk_error_string(int code) {
  switch (code) {
    case QMK_OK: return "ok";
    case QMK_ERR_ARGS: return "invalid argument";
    case QMK_ERR_CUDA: return "CUDA runtime error";
    case QMK_ERR_LAUNCH: return "cooperative launch refused";
    case QMK_ERR_TIMEOUT: return "device-side wait timed out";
    case QMK_ERR_TOKEN: return "token id out of range";
    case QMK_ERR_WORKSPACE: return "workspace too small or misaligned";
    default: return "unknown error";
  }
}

int qmk_get_last_error(void) { return g_last_error; }
const char *qmk_get_last_error_message(void) { return g_last_msg; }

int qmk_attention_splits(int num_ctas, int max_position) {
  return qmk::attention_splits(num_ctas, max_position);
}

int qmk_describe_partition(int num_ctas, int splits, int cta, int *out, int out_len) {
  if (!out || out_len < 12 || num_ctas < qmk::kMinCtas || num_ctas > qmk::kMaxCtas || cta < 0 ||
      cta >= num_ctas || splits < 1 || splits > qmk::kMaxSplits || qmk::kNumKVHeads * splits > num_ctas)
    return set_error(QMK_ERR_ARGS, "qmk_describe_partition: bad arguments");
  const qmk::Range a = qmk::qkv_rows(cta, num_ctas), b = qmk::o_rows(cta, num_ctas),
                   g = qmk::gu_rows(cta, num_ctas), d = qmk::d_rows(cta, num_ctas),
                   lm = qmk::lm_rows(cta, num_ctas);
  out[0] = a.begin; out[1] = a.end;
  out[2] = b.begin; out[3] = b.end;
  out[4] = g.begin; out[5] = g.end;
  out[6] = d.begin; out[7] = d.end;
  out[8] = lm.begin; out[9] = lm.end;
  out[10] = qmk::item_of_cta(cta, splits);
  out[11] = qmk::merge_task_of_cta(cta, num_ctas);
  return clear_error();
}

int qmk_num_ctas(int device) {
  int sms = 0;
  cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) {
    set_error(QMK_ERR_CUDA, "SM count: %s", cudaGetErrorString(e));
    return -1;
  }
  return sms < qmk::kMaxCtas ? sms : qmk::kMaxCtas;
}

int qmk_workspace_init(void *workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (!workspace || workspace_bytes < (size_t)qmk::kWorkspaceBytes || !aligned(workspace, 256))
    return set_error(QMK_ERR_WORKSPACE, "workspace needs %lld bytes, 256-byte aligned",
                     (long long)qmk::kWorkspaceBytes);
  cudaError_t e = cudaMemsetAsync(workspace, 0, (size_t)qmk::kWorkspaceBytes, stream);
  if (e != cudaSuccess) return set_error(QMK_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  return clear_error();
}

int qmk_run(const QmkRunArgs *a, cudaStream_t stream) {
  if (!a) return set_error(QMK_ERR_ARGS, "qmk_run: null args");
  if (!a->embed_weight || !a->layer_weights || !a->final_norm_weight || !a->lm_head_weight ||
      !a->cos_table || !a->sin_table || !a->k_cache || !a->v_cache)
    return set_error(QMK_ERR_ARGS, "qmk_run: null weight/table/cache pointer");
  if (!a->workspace || a->workspace_bytes < (size_t)qmk::kWorkspaceBytes || !aligned(a->workspace, 256))
    return set_error(QMK_ERR_WORKSPACE, "qmk_run: workspace needs %lld bytes, 256-byte aligned",
                     (long long)qmk::kWorkspaceBytes);
  if (a->num_layers < 1 || a->num_layers > qmk::kMaxLayers)
    return set_error(QMK_ERR_ARGS, "qmk_run: num_layers=%d outside [1, %d]", a->num_layers, qmk::kMaxLayers);
  if (a->num_steps < 1) return set_error(QMK_ERR_ARGS, "qmk_run: num_steps=%d < 1", a->num_steps);
  if (a->max_seq_len < 1) return set_error(QMK_ERR_ARGS, "qmk_run: max_seq_len=%d < 1", a->max_seq_len);
  if (a->start_position < 0 || (long long)a->start_position + a->num_steps > a->max_seq_len)
    return set_error(QMK_ERR_ARGS,
                     "qmk_run: positions [%d, %lld) exceed max_seq_len=%d", a->start_position,
                     (long long)a->start_position + a->num_steps, a->max_seq_len);
  if ((long long)a->num_steps * (a->num_layers + 1) >= (1LL << 27))
    return set_error(QMK_ERR_ARGS, "qmk_run: num_steps=%d too large for one launch", a->num_steps);
  if (a->n_forced < 0 || (a->n_forced > 0 && !a->forced_tokens))
    return set_error(QMK_ERR_ARGS, "qmk_run: n_forced=%d without forced_tokens", a->n_forced);
  if (a->n_forced == 0 && (a->first_token < 0 || a->first_token >= QMK_VOCAB))
    return set_error(QMK_ERR_ARGS, "qmk_run: token id %d outside [0, %d)", a->first_token, QMK_VOCAB);
  if (!(a->attn_scale == a->attn_scale) || a->attn_scale <= 0.f)
    return set_error(QMK_ERR_ARGS, "qmk_run: attn_scale must be positive");
  if (!(a->temperature >= 0.f) || a->temperature > 1e30f)
    return set_error(QMK_ERR_ARGS, "qmk_run: temperature must be finite and >= 0");
  if (a->top_k < 0 || a->top_k > qmk::kMaxTopK)
    return set_error(QMK_ERR_ARGS, "qmk_run: top_k=%d outside [0, %d]", a->top_k, qmk::kMaxTopK);
  if (a->stop_at_eos && (a->eos_token < 0 || a->eos_token >= QMK_VOCAB))
    return set_error(QMK_ERR_ARGS, "qmk_run: eos_token %d outside [0, %d)", a->eos_token, QMK_VOCAB);
  const void *ptrs[] = {a->embed_weight, a->final_norm_weight, a->lm_head_weight, a->cos_table,
                        a->sin_table,    a->k_cache,           a->v_cache};
  for (const void *q : ptrs)
    if (!aligned(q, 16)) return set_error(QMK_ERR_ARGS, "qmk_run: tensor not 16-byte aligned");
  if (!aligned(a->layer_weights, 8)) return set_error(QMK_ERR_ARGS, "qmk_run: layer table misaligned");

  int dev = 0;
  if (current_device(&dev) != QMK_OK) return g_last_error;
  int ncta;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (prepare_device(dev) != QMK_OK) return g_last_error;
    ncta = g_devices[dev].num_sms;
  }
  if (ncta > qmk::kMaxCtas) ncta = qmk::kMaxCtas;
  // top-k keeps a CTA's LM-head logits in 2048 floats of shared memory
  if (a->top_k > 0 && (qmk::kVocab + ncta - 1) / ncta > 2 * qmk::kHidden)
    return set_error(QMK_ERR_ARGS, "qmk_run: top_k needs at least %d SMs", (qmk::kVocab + 2 * qmk::kHidden - 1) / (2 * qmk::kHidden));
  if (ncta < qmk::kMinCtas)
    return set_error(QMK_ERR_LAUNCH, "qmk_run: %d SMs < %d required", ncta, qmk::kMinCtas);

  qmk::Params p;
  p.embed = (const __nv_bfloat16 *)a->embed_weight;
  p.layers = a->layer_weights;
  p.final_norm = (const __nv_bfloat16 *)a->final_norm_weight;
  p.lm_head = (const __nv_bfloat16 *)a->lm_head_weight;
  p.cos_t = (const __nv_bfloat16 *)a->cos_table;
  p.sin_t = (const __nv_bfloat16 *)a->sin_table;
  p.k_cache = (__nv_bfloat16 *)a->k_cache;
  p.v_cache = (__nv_bfloat16 *)a->v_cache;
  p.ws = (uint8_t *)a->workspace;
  p.forced = a->forced_tokens;
  p.n_forced = a->n_forced < a->num_steps ? a->n_forced : a->num_steps;
  p.first_token = a->first_token;
  p.start_pos = a->start_position;
  p.num_steps = a->num_steps;
  p.num_layers = a->num_layers;
  p.max_seq_len = a->max_seq_len;
  p.attn_scale = a->attn_scale;
  p.splits = qmk::attention_splits(ncta, a->start_position + a->num_steps - 1);
  p.out_log = a->output_log;
  p.out_token = a->output_token;
  p.logits = a->logits;
  p.final_hidden = a->final_hidden;
  p.status = a->status;
  p.timeout_ns = a->timeout_ns ? a->timeout_ns : qmk::kDefaultTimeoutNs;
  p.debug_stall = (a->debug_stall > 0 && a->debug_stall <= ncta) ? a->debug_stall : 0;
  p.trace = a->trace;
  p.trace_step = a->trace_step;
  p.poll_backoff_ns = a->poll_backoff_ns > 4096u ? 4096u : a->poll_backoff_ns;
  p.tuning = a->tuning;
  p.inv_temp = a->temperature > 0.f ? 1.0f / a->temperature : 0.f;
  p.seed = a->seed;
  p.eos_token = a->stop_at_eos ? a->eos_token : -1;
  p.top_k = a->top_k;
  p.steps_done = a->steps_done;

  void *kargs[] = {&p};
  // the feature instance only when a feature is asked for
  const bool feat = p.top_k > 0 || p.inv_temp > 0.f || p.trace || p.tuning || p.poll_backoff_ns;
  const void *kernel = feat ? (const void *)qmk::decode_kernel<true> : (const void *)qmk::decode_kernel<false>;
  cudaError_t e = cudaLaunchCooperativeKernel(kernel, dim3(ncta),
                                              dim3(qmk::kThreads), kargs, qmk::kSmBytes, stream);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(e == cudaErrorCooperativeLaunchTooLarge ? QMK_ERR_LAUNCH : QMK_ERR_CUDA,
                     "cooperative launch of %d x %d: %s", ncta, qmk::kThreads, cudaGetErrorString(e));
  }
  return clear_error();
}

static_assert(qmk::kBatchSeqs == QMK_BATCH_SEQS, "batched sequence count");

int qmk_run_batch(const QmkBatchRunArgs *a, cudaStream_t stream) {
  constexpr int NB = qmk::kBatchSeqs;
  if (!a) return set_error(QMK_ERR_ARGS, "qmk_run_batch: null args");
  if (!a->embed_weight || !a->layer_weights || !a->final_norm_weight || !a->lm_head_weight || !a->cos_table ||
      !a->sin_table || !a->k_cache || !a->v_cache || !a->workspace || !a->first_tokens)
    return set_error(QMK_ERR_ARGS, "qmk_run_batch: null pointer argument");
  if (a->workspace_bytes < (size_t)qmk::kWorkspaceBytes)
    return set_error(QMK_ERR_WORKSPACE, "qmk_run_batch: workspace %zu < %lld bytes", a->workspace_bytes,
                     (long long)qmk::kWorkspaceBytes);
  if (!aligned(a->workspace, 256)) return set_error(QMK_ERR_WORKSPACE, "qmk_run_batch: workspace misaligned");
  if (a->num_layers < 1 || a->num_layers > qmk::kMaxLayers)
    return set_error(QMK_ERR_ARGS, "qmk_run_batch: num_layers=%d outside [1, %d]", a->num_layers, qmk::kMaxLayers);
  if (a->num_steps < 1) return set_error(QMK_ERR_ARGS, "qmk_run_batch: num_steps=%d", a->num_steps);
  if (a->max_seq_len < 1) return set_error(QMK_ERR_ARGS, "qmk_run_batch: max_seq_len=%d", a->max_seq_len);
  if (a->cache_seq_stride < (long long)a->num_layers * qmk::kNumKVHeads * a->max_seq_len * qmk::kHeadDim ||
      a->cache_seq_stride % 8)
    return set_error(QMK_ERR_ARGS, "qmk_run_batch: cache_seq_stride %lld too small or not 16-byte aligned",
                     a->cache_seq_stride);
  int max_pos = 0;
  for (int b = 0; b < NB; ++b) {
    const int s0 = a->start_positions[b];
    if (s0 < 0 || (long long)s0 + a->num_steps > a->max_seq_len)
      return set_error(QMK_ERR_ARGS, "qmk_run_batch: sequence %d: positions [%d, %d) outside [0, %d)", b, s0,
                       s0 + a->num_steps, a->max_seq_len);
    if (s0 + a->num_steps - 1 > max_pos) max_pos = s0 + a->num_steps - 1;
  }
  if (!(a->attn_scale == a->attn_scale) || a->attn_scale <= 0.f)
    return set_error(QMK_ERR_ARGS, "qmk_run_batch: attn_scale must be positive");
  const void *ptrs[] = {a->embed_weight, a->final_norm_weight, a->lm_head_weight, a->cos_table,
                        a->sin_table,    a->k_cache,           a->v_cache};
  for (const void *q : ptrs)
    if (!aligned(q, 16)) return set_error(QMK_ERR_ARGS, "qmk_run_batch: tensor not 16-byte aligned");
  if (!aligned(a->layer_weights, 8)) return set_error(QMK_ERR_ARGS, "qmk_run_batch: layer table misaligned");

  int dev = 0;
  if (current_device(&dev) != QMK_OK) return g_last_error;
  int ncta;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (prepare_device(dev) != QMK_OK) return g_last_error;
    ncta = g_devices[dev].num_sms;
  }
  if (ncta > qmk::kMaxCtas) ncta = qmk::kMaxCtas;
  // attention items (NB x 8 KV heads) and merge tasks (NB x 32) one per CTA;
  // O / down rows per CTA within the residual slots
  if (ncta < NB * qmk::kMergeTasks || (qmk::kHidden + ncta - 1) / ncta > qmk::kMaxResRows || ncta < qmk::kMinCtas)
    return set_error(QMK_ERR_LAUNCH, "qmk_run_batch: %d SMs < %d required", ncta, NB * qmk::kMergeTasks);

  qmk::Params p;
  memset(&p, 0, sizeof(p));
  p.embed = (const __nv_bfloat16 *)a->embed_weight;
  p.layers = a->layer_weights;
  p.final_norm = (const __nv_bfloat16 *)a->final_norm_weight;
  p.lm_head = (const __nv_bfloat16 *)a->lm_head_weight;
  p.cos_t = (const __nv_bfloat16 *)a->cos_table;
  p.sin_t = (const __nv_bfloat16 *)a->sin_table;
  p.k_cache = (__nv_bfloat16 *)a->k_cache;
  p.v_cache = (__nv_bfloat16 *)a->v_cache;
  p.ws = (uint8_t *)a->workspace;
  p.num_steps = a->num_steps;
  p.num_layers = a->num_layers;
  p.max_seq_len = a->max_seq_len;
  p.attn_scale = a->attn_scale;
  p.splits = qmk::attention_splits(ncta, max_pos, NB);
  p.out_log = a->output_log;
  p.status = a->status;
  p.timeout_ns = a->timeout_ns ? a->timeout_ns : qmk::kDefaultTimeoutNs;
  p.eos_token = -1;
  for (int b = 0; b < NB; ++b) p.start_pos_b[b] = a->start_positions[b];
  p.start_pos = a->start_positions[0];
  p.cache_seq_stride = a->cache_seq_stride;
  p.first_tokens_b = a->first_tokens;

  void *kargs[] = {&p};
  cudaError_t e = cudaLaunchCooperativeKernel((const void *)qmk::decode_kernel<false, NB>, dim3(ncta),
                                              dim3(qmk::kThreads), kargs, qmk::kSmBytes, stream);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(e == cudaErrorCooperativeLaunchTooLarge ? QMK_ERR_LAUNCH : QMK_ERR_CUDA,
                     "cooperative launch of %d x %d: %s", ncta, qmk::kThreads, cudaGetErrorString(e));
  }
  return clear_error();
}

// ---- library-owned default workspace (reference entry points) ----

static int default_state(DeviceState **out) {
  int dev = 0;
  if (current_device(&dev) != QMK_OK) return g_last_error;
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceState &ds = g_devices[dev];
  if (!ds.default_ws) {
    void *ws = nullptr;
    cudaError_t e = cudaMalloc(&ws, (size_t)qmk::kWorkspaceBytes);
    if (e != cudaSuccess) return set_error(QMK_ERR_CUDA, "cudaMalloc(workspace): %s", cudaGetErrorString(e));
    e = cudaMemset(ws, 0, (size_t)qmk::kWorkspaceBytes);
    if (e != cudaSuccess) return set_error(QMK_ERR_CUDA, "cudaMemset(workspace): %s", cudaGetErrorString(e));
    void *host = nullptr;
    e = cudaHostAlloc(&host, sizeof(QmkStatus), cudaHostAllocMapped);
    if (e != cudaSuccess) return set_error(QMK_ERR_CUDA, "cudaHostAlloc(status): %s", cudaGetErrorString(e));
    memset(host, 0, sizeof(QmkStatus));
    void *devp = nullptr;
    e = cudaHostGetDevicePointer(&devp, host, 0);
    if (e != cudaSuccess) return set_error(QMK_ERR_CUDA, "cudaHostGetDevicePointer: %s", cudaGetErrorString(e));
    ds.default_ws = ws;
    ds.default_status_host = (QmkStatus *)host;
    ds.default_status_dev = (QmkStatus *)devp;
  }
  *out = &ds;
  return QMK_OK;
}

int qmk_read_default_status(QmkStatus *out) {
  if (!out) return set_error(QMK_ERR_ARGS, "qmk_read_default_status: null");
  DeviceState *ds = nullptr;
  if (default_state(&ds) != QMK_OK) return g_last_error;
  const volatile QmkStatus *st = ds->default_status_host;
  out->error_code = st->error_code;
  out->error_info = st->error_info;
  out->launches = st->launches;
  out->epoch = st->epoch;
  return clear_error();
}

static void reference_launch(int first_token, int num_steps, const void *embed_weight,
                             const LDGLayerWeights *layer_weights, const void *final_norm_weight,
                             const void *lm_head_weight, const void *cos_table, const void *sin_table,
                             void *k_cache, void *v_cache, void *g_normalized, int *output_log,
                             int *output_token, int num_layers, int start_position, int max_seq_len,
                             float attn_scale, cudaStream_t stream) {
  DeviceState *ds = nullptr;
  if (default_state(&ds) != QMK_OK) return;
  QmkRunArgs a;
  memset(&a, 0, sizeof(a));
  a.embed_weight = embed_weight;
  a.layer_weights = layer_weights;
  a.final_norm_weight = final_norm_weight;
  a.lm_head_weight = lm_head_weight;
  a.cos_table = cos_table;
  a.sin_table = sin_table;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.workspace = ds->default_ws;
  a.workspace_bytes = (size_t)qmk::kWorkspaceBytes;
  a.first_token = first_token;
  a.start_position = start_position;
  a.num_steps = num_steps;
  a.num_layers = num_layers;
  a.max_seq_len = max_seq_len;
  a.attn_scale = attn_scale;
  a.output_log = output_log;
  a.output_token = output_token;
  a.final_hidden = (float *)g_normalized;
  a.status = ds->default_status_dev;
  qmk_run(&a, stream);
}

void launch_ldg_decode_direct(int input_token_id, int *output_token_id, const void *embed_weight,
                              const LDGLayerWeights *layer_weights, const void *final_norm_weight,
                              const void *lm_head_weight, const void *cos_table, const void *sin_table,
                              void *k_cache, void *v_cache, void *hidden_buffer, void *g_activations,
                              void *g_residual, void *g_q, void *g_k, void *g_v, void *g_attn_out,
                              void *g_mlp_intermediate, void *g_normalized, void *block_max_vals,
                              void *block_max_idxs, int num_layers, int position, int max_seq_len,
                              float attn_scale, cudaStream_t stream) {
  (void)hidden_buffer; (void)g_activations; (void)g_residual; (void)g_q; (void)g_k; (void)g_v;
  (void)g_attn_out; (void)g_mlp_intermediate; (void)block_max_vals; (void)block_max_idxs;
  reference_launch(input_token_id, 1, embed_weight, layer_weights, final_norm_weight, lm_head_weight,
                   cos_table, sin_table, k_cache, v_cache, g_normalized, nullptr, output_token_id,
                   num_layers, position, max_seq_len, attn_scale, stream);
}

void launch_ldg_decode_persistent(int input_token_id, int *output_token_id, const void *embed_weight,
                                  const LDGLayerWeights *layer_weights, const void *final_norm_weight,
                                  const void *lm_head_weight, const void *cos_table,
                                  const void *sin_table, void *k_cache, void *v_cache,
                                  void *hidden_buffer, void *g_activations, void *g_residual, void *g_q,
                                  void *g_k, void *g_v, void *g_attn_out, void *g_mlp_intermediate,
                                  void *g_normalized, void *block_max_vals, void *block_max_idxs,
                                  int num_layers, int position, int cache_len, int max_seq_len,
                                  float attn_scale, cudaStream_t stream) {
  (void)cache_len;
  launch_ldg_decode_direct(input_token_id, output_token_id, embed_weight, layer_weights,
                           final_norm_weight, lm_head_weight, cos_table, sin_table, k_cache, v_cache,
                           hidden_buffer, g_activations, g_residual, g_q, g_k, g_v, g_attn_out,
                           g_mlp_intermediate, g_normalized, block_max_vals, block_max_idxs,
                           num_layers, position, max_seq_len, attn_scale, stream);
}

void launch_ldg_generate_nosync(int first_token_id, int num_steps, const void *embed_weight,
                                const LDGLayerWeights *layer_weights, const void *final_norm_weight,
                                const void *lm_head_weight, const void *cos_table, const void *sin_table,
                                void *k_cache, void *v_cache, void *hidden_buffer, void *g_activations,
                                void *g_residual, void *g_q, void *g_k, void *g_v, void *g_attn_out,
                                void *g_mlp_intermediate, void *g_normalized, void *block_max_vals,
                                void *block_max_idxs, int *output_log, int num_layers,
                                int start_position, int max_seq_len, float attn_scale,
                                cudaStream_t stream) {
  (void)hidden_buffer; (void)g_activations; (void)g_residual; (void)g_q; (void)g_k; (void)g_v;
  (void)g_attn_out; (void)g_mlp_intermediate; (void)block_max_vals; (void)block_max_idxs;
  reference_launch(first_token_id, num_steps, embed_weight, layer_weights, final_norm_weight,
                   lm_head_weight, cos_table, sin_table, k_cache, v_cache, g_normalized, output_log,
                   nullptr, num_layers, start_position, max_seq_len, attn_scale, stream);
}

// ---- allocation-free variant: file-scope static scratch ----

}  // extern "C"

namespace {

// Scratch of qmk_generate_static: [workspace | token log | status].
constexpr size_t kStaticLogOff = (size_t)qmk::kWorkspaceBytes;
constexpr size_t kStaticStatusOff = kStaticLogOff + 4 * (size_t)QMK_STATIC_MAX_STEPS;
static_assert(kStaticStatusOff + 256 <= (size_t)QMK_STATIC_SCRATCH_BYTES, "static scratch too small");
static_assert(kStaticLogOff % 256 == 0, "token log alignment");

__device__ __align__(256) unsigned char g_static_scratch[QMK_STATIC_SCRATCH_BYTES];

uint8_t *g_static_ptr[kMaxDevices] = {};

// Device address of g_static_scratch on the current device (looked up once).
int static_scratch(uint8_t **out) {
  int dev = 0;
  if (current_device(&dev) != QMK_OK) return g_last_error;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_static_ptr[dev]) {
    void *ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_static_scratch);
    if (e != cudaSuccess || !ptr)
      return set_error(QMK_ERR_CUDA, "cudaGetSymbolAddress(static scratch) on device %d: %s", dev,
                       cudaGetErrorString(e));
    g_static_ptr[dev] = static_cast<uint8_t *>(ptr);
  }
  *out = g_static_ptr[dev];
  return QMK_OK;
}

}  // namespace

extern "C" {

int qmk_generate_static(int first_token_id, int num_steps, const void *embed_weight,
                        const LDGLayerWeights *layer_weights, const void *final_norm_weight,
                        const void *lm_head_weight, const void *cos_table, const void *sin_table,
                        void *k_cache, void *v_cache, int num_layers, int start_position,
                        int max_seq_len, float attn_scale, cudaStream_t stream) {
  if (num_steps < 1 || num_steps > QMK_STATIC_MAX_STEPS)
    return set_error(QMK_ERR_ARGS,
                     "qmk_generate_static: num_steps=%d outside [1, %d] (capacity of the static token log)",
                     num_steps, QMK_STATIC_MAX_STEPS);
  uint8_t *base = nullptr;
  if (static_scratch(&base) != QMK_OK) return g_last_error;
  QmkRunArgs a;
  memset(&a, 0, sizeof(a));
  a.embed_weight = embed_weight;
  a.layer_weights = layer_weights;
  a.final_norm_weight = final_norm_weight;
  a.lm_head_weight = lm_head_weight;
  a.cos_table = cos_table;
  a.sin_table = sin_table;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.workspace = base;
  a.workspace_bytes = (size_t)qmk::kWorkspaceBytes;
  a.first_token = first_token_id;
  a.start_position = start_position;
  a.num_steps = num_steps;
  a.num_layers = num_layers;
  a.max_seq_len = max_seq_len;
  a.attn_scale = attn_scale;
  a.output_log = reinterpret_cast<int *>(base + kStaticLogOff);
  a.status = reinterpret_cast<QmkStatus *>(base + kStaticStatusOff);
  return qmk_run(&a, stream);
}

int qmk_static_scratch_ptrs(int **output_log, QmkStatus **status) {
  uint8_t *base = nullptr;
  if (static_scratch(&base) != QMK_OK) return g_last_error;
  if (output_log) *output_log = reinterpret_cast<int *>(base + kStaticLogOff);
  if (status) *status = reinterpret_cast<QmkStatus *>(base + kStaticStatusOff);
  return clear_error();
}

}  // extern "C"
