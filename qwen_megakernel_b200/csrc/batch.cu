// Token-parallel forward pass (prefill of a prompt, batched decode of several
// sequences) for Qwen3-0.6B on sm_100a.  Entry point: qmk_batch_forward
// (include/qwen_megakernel.h).
//
// The decode megakernel streams every weight once per token; with M rows in
// flight the projections become GEMMs [M, K] x [K, N] that reuse each weight
// M times, so they go to the tensor cores through cuBLAS (plain GEMMs, bf16
// operands, fp32 accumulation).  The fp32 activations are fed as a bf16 pair
// x = hi + lo (lo = rounding remainder of hi): two GEMMs per projection keep
// the products exact and the activation error at ~2^-17, the precision the
// decode kernel keeps, so both paths agree with the fp32 oracle within the
// same tolerance.  Everything between the GEMMs is fused into one kernel per
// step: RMSNorm + split, QK-norm + RoPE + K/V append, attention (+ split of
// its output), SiLU(gate) * up (+ split), final norm + argmax.
//
// Reference steps these kernels restate (AlpinDale/qwen_megakernel):
//   RMSNorm eps 1e-6              csrc/kernel.cu:168-292 (ldg_matvec_qkv)
//   QK-norm, RoPE, K/V append     csrc/kernel.cu:316-400
//   GQA attention, online softmax csrc/kernel.cu:400-643
//   O-proj + residual, post-norm, SiLU(gate) * up, down + residual
//                                 csrc/kernel.cu:649-865
//   final norm, LM head, argmax   csrc/kernel.cu:1020-1183, 1386-1423

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "qmk_device.cuh"
#include "qwen_megakernel.h"

int qmk_internal_set_error(int code, const char *msg);
int qmk_internal_clear_error();

namespace qmb {

constexpr int kHidden = QMK_HIDDEN;
constexpr int kInter = QMK_INTERMEDIATE;
constexpr int kHeadDim = QMK_HEAD_DIM;
constexpr int kNumQHeads = QMK_NUM_Q_HEADS;
constexpr int kNumKVHeads = QMK_NUM_KV_HEADS;
constexpr int kQSize = kNumQHeads * kHeadDim;    // 2048
constexpr int kKVSize = kNumKVHeads * kHeadDim;  // 1024
constexpr int kQKV = kQSize + 2 * kKVSize;       // 4096
constexpr int kVocab = QMK_VOCAB;
constexpr float kRmsEps = 1e-6f;
constexpr float kLog2e = 1.4426950408889634f;

using qmk::pdl_trigger;
using qmk::pdl_wait;

__device__ __forceinline__ float bf_lo(unsigned u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(unsigned u) { return __uint_as_float(u & 0xffff0000u); }

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

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// v ~= hi + lo with hi = bf16(v), lo = bf16(v - hi): four elements at once.
__device__ __forceinline__ void split4(const float (&v)[4], uint2 &hi, uint2 &lo) {
  const __nv_bfloat162 h0 = __floats2bfloat162_rn(v[0], v[1]);
  const __nv_bfloat162 h1 = __floats2bfloat162_rn(v[2], v[3]);
  const float2 f0 = __bfloat1622float2(h0), f1 = __bfloat1622float2(h1);
  const __nv_bfloat162 l0 = __floats2bfloat162_rn(v[0] - f0.x, v[1] - f0.y);
  const __nv_bfloat162 l1 = __floats2bfloat162_rn(v[2] - f1.x, v[3] - f1.y);
  hi = make_uint2(*reinterpret_cast<const unsigned *>(&h0), *reinterpret_cast<const unsigned *>(&h1));
  lo = make_uint2(*reinterpret_cast<const unsigned *>(&l0), *reinterpret_cast<const unsigned *>(&l1));
}

// Block (256 threads) sum; every thread gets the total.  red: 8 floats.
__device__ __forceinline__ float block_sum256(float v, float *red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5;
  __syncthreads();  // red may still be read by a previous call
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) t += red[i];
  return t;
}

// ---------------------------------------------------------------- kernels
// x[r] = embed[tokens[r]] (bf16 -> fp32).  Grid: rows, 256 threads, 4 each.
__global__ void __launch_bounds__(256) embed_kernel(const __nv_bfloat16 *__restrict__ embed,
                                                   const int *__restrict__ tokens, float *__restrict__ x,
                                                   unsigned *status) {
  pdl_wait();  // inputs are written by the previous kernel
  pdl_trigger();
  const int r = blockIdx.x;
  int tok = tokens[r];
  if (tok < 0 || tok >= kVocab) {
    if (threadIdx.x == 0 && status) atomicOr(status, QMK_BATCH_BAD_TOKEN);
    tok = 0;
  }
  const uint2 v = __ldg(reinterpret_cast<const uint2 *>(embed + (size_t)tok * kHidden) + threadIdx.x);
  reinterpret_cast<float4 *>(x + (size_t)r * kHidden)[threadIdx.x] =
      make_float4(bf_lo(v.x), bf_hi(v.x), bf_lo(v.y), bf_hi(v.y));
}

// Residual add + RMSNorm (eps 1e-6) times w, split into the bf16 GEMM input.
// GEMM inputs and outputs are "stacked": for n rows the hi halves fill rows
// [0, n) and the lo halves rows [n, 2n), so ONE GEMM over 2n rows reads each
// weight once for both halves; the consumer of its fp32 output adds row r
// and row n + r.  Here: v = x[r] + sum over the nsplit K-split partials c of
// (c[r] + c[num_in + r]) (c = c2 + s split_stride: the stacked output of the
// previous projection, or c2 null), with r = rows ? rows[i] : i;
// without `rows` v is written back to x (the residual stream).  Output row i
// of n_out = gridDim.x: hi at a2 row i, lo at a2 row n_out + i (stride 1024).
__global__ void __launch_bounds__(256) residual_norm_split_kernel(float *__restrict__ x,
                                                                  const float *__restrict__ c2,
                                                                  const int *__restrict__ rows, int num_in,
                                                                  const __nv_bfloat16 *__restrict__ w,
                                                                  __nv_bfloat16 *__restrict__ a2, int nsplit,
                                                                  long long split_stride) {
  pdl_wait();  // inputs are written by the previous kernel
  pdl_trigger();
  __shared__ float red[8];
  const int i = blockIdx.x, n_out = gridDim.x;
  int r = rows ? rows[i] : i;
  if (r < 0 || r >= num_in) r = 0;  // validated on the host; never read out of bounds
  float4 v = reinterpret_cast<const float4 *>(x + (size_t)r * kHidden)[threadIdx.x];
  if (c2) {
    // nsplit K-split partial products of the GEMM, each stacked hi/lo
    float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sp = 0; sp < nsplit; ++sp) {
      const float *c = c2 + (size_t)sp * (size_t)split_stride;
      const float4 h = reinterpret_cast<const float4 *>(c + (size_t)r * kHidden)[threadIdx.x];
      const float4 l = reinterpret_cast<const float4 *>(c + (size_t)(num_in + r) * kHidden)[threadIdx.x];
      sum.x += h.x + l.x;
      sum.y += h.y + l.y;
      sum.z += h.z + l.z;
      sum.w += h.w + l.w;
    }
    v.x += sum.x;
    v.y += sum.y;
    v.z += sum.z;
    v.w += sum.w;
    if (!rows) reinterpret_cast<float4 *>(x + (size_t)r * kHidden)[threadIdx.x] = v;
  }
  const float ss = block_sum256(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w, red);
  const float rstd = rsqrtf(ss / (float)kHidden + kRmsEps);
  const uint2 wv = __ldg(reinterpret_cast<const uint2 *>(w) + threadIdx.x);
  const float y[4] = {v.x * rstd * bf_lo(wv.x), v.y * rstd * bf_hi(wv.x), v.z * rstd * bf_lo(wv.y),
                      v.w * rstd * bf_hi(wv.y)};
  uint2 h, l;
  split4(y, h, l);
  reinterpret_cast<uint2 *>(a2 + (size_t)i * kHidden)[threadIdx.x] = h;
  reinterpret_cast<uint2 *>(a2 + (size_t)(n_out + i) * kHidden)[threadIdx.x] = l;
}

// Per-head RMSNorm of q and k (weights [128]) of the stacked QKV GEMM output
// [2 rows, 4096] (nsplit K-split partials split_stride floats apart), RoPE (rotate-half, bf16 tables) at the row's position, K/V rounded to bf16 into the sequence's
// cache, q scaled by attn_scale * log2(e) (scores in log2 units).  Grid:
// rows, 256 threads: warp w takes q heads w and w + 8, K/V head w; lane l
// holds dims 4l .. 4l + 3, the rotation partner (d +- 64) sits in lane l ^ 16.
__global__ void __launch_bounds__(256) qk_rope_kv_kernel(
    const float *__restrict__ qkv, const __nv_bfloat16 *__restrict__ q_norm,
    const __nv_bfloat16 *__restrict__ k_norm, const __nv_bfloat16 *__restrict__ cos_t,
    const __nv_bfloat16 *__restrict__ sin_t, const int *__restrict__ row_seq, const int *__restrict__ row_pos,
    __nv_bfloat16 *__restrict__ k_cache, __nv_bfloat16 *__restrict__ v_cache, long long kv_seq_stride,
    int num_seqs, int layer, int max_seq_len, float q_scale, float *__restrict__ q_out, unsigned *status,
    int nsplit, long long split_stride) {
  pdl_wait();  // inputs are written by the previous kernel
  pdl_trigger();
  const int r = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int seq = row_seq[r], pos = row_pos[r];
  if (seq < 0 || seq >= num_seqs || pos < 0 || pos >= max_seq_len) {
    if (threadIdx.x == 0 && status) atomicOr(status, QMK_BATCH_BAD_ROW);
    return;
  }
  const int d0 = 4 * lane;
  const uint2 cv = __ldg(reinterpret_cast<const uint2 *>(cos_t + (size_t)pos * kHeadDim + d0));
  const uint2 sv = __ldg(reinterpret_cast<const uint2 *>(sin_t + (size_t)pos * kHeadDim + d0));
  const float cf[4] = {bf_lo(cv.x), bf_hi(cv.x), bf_lo(cv.y), bf_hi(cv.y)};
  const float sf[4] = {bf_lo(sv.x), bf_hi(sv.x), bf_lo(sv.y), bf_hi(sv.y)};
  const float *row = qkv + (size_t)r * kQKV;
  const float *row_lo = qkv + (size_t)(gridDim.x + r) * kQKV;  // stacked GEMM output: hi + lo rows
  auto load4 = [&](int col) {  // hi + lo rows of every K-split partial, in split order
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sp = 0; sp < nsplit; ++sp) {
      const size_t o = (size_t)sp * (size_t)split_stride;
      const float4 h = *reinterpret_cast<const float4 *>(row + o + col);
      const float4 l = *reinterpret_cast<const float4 *>(row_lo + o + col);
      acc.x += h.x + l.x;
      acc.y += h.y + l.y;
      acc.z += h.z + l.z;
      acc.w += h.w + l.w;
    }
    return acc;
  };
  auto norm_rope = [&](int col, const __nv_bfloat16 *nw, float (&y)[4]) {
    const float4 x4 = load4(col + d0);
    float x[4] = {x4.x, x4.y, x4.z, x4.w};
    const float rr = rsqrtf(warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]) / (float)kHeadDim + kRmsEps);
    const uint2 wv = __ldg(reinterpret_cast<const uint2 *>(nw + d0));
    const float wf[4] = {bf_lo(wv.x), bf_hi(wv.x), bf_lo(wv.y), bf_hi(wv.y)};
#pragma unroll
    for (int e = 0; e < 4; ++e) x[e] = (x[e] * rr) * wf[e];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float partner = __shfl_xor_sync(0xffffffffu, x[e], 16);
      y[e] = (lane < 16) ? (x[e] * cf[e] - partner * sf[e]) : (x[e] * cf[e] + partner * sf[e]);
    }
  };
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int h = warp + 8 * k;
    float y[4];
    norm_rope(h * kHeadDim, q_norm, y);
    *reinterpret_cast<float4 *>(q_out + (size_t)r * kQSize + h * kHeadDim + d0) =
        make_float4(y[0] * q_scale, y[1] * q_scale, y[2] * q_scale, y[3] * q_scale);
  }
  float ky[4];
  norm_rope(kQSize + warp * kHeadDim, k_norm, ky);
  const float4 v4 = load4(kQSize + kKVSize + warp * kHeadDim + d0);
  const size_t off = (size_t)seq * (size_t)kv_seq_stride +
                     (((size_t)layer * kNumKVHeads + warp) * (size_t)max_seq_len + pos) * kHeadDim + d0;
  const __nv_bfloat162 k01 = __floats2bfloat162_rn(ky[0], ky[1]), k23 = __floats2bfloat162_rn(ky[2], ky[3]);
  const __nv_bfloat162 v01 = __floats2bfloat162_rn(v4.x, v4.y), v23 = __floats2bfloat162_rn(v4.z, v4.w);
  *reinterpret_cast<uint2 *>(k_cache + off) =
      make_uint2(*reinterpret_cast<const unsigned *>(&k01), *reinterpret_cast<const unsigned *>(&k23));
  *reinterpret_cast<uint2 *>(v_cache + off) =
      make_uint2(*reinterpret_cast<const unsigned *>(&v01), *reinterpret_cast<const unsigned *>(&v23));
}

// GQA attention of row r over positions [0, row_pos[r]] of its sequence's
// cache for the q heads 2g, 2g+1 of KV head g (grid (g, r, split), 256
// threads; split s of `splits` takes the s-th of equal position chunks, so
// small batches still fill the GPU).
// The chunk streams through shared memory: 64-position tiles (K rows, then
// V rows, 16 KB each) in a kAttStages-deep ring of 1-D bulk copies issued by
// thread 0 and completed on one mbarrier per stage, so several tiles per CTA
// are in flight while the warps work on an earlier one (direct loads left
// the kernel waiting on HBM latency with one tile in flight).
// Group gq = lane / 8 of a warp takes one position per round; lane r8 of
// the group holds dims [8 r8, 8 r8 + 8) and [64 + 8 r8, 64 + 8 r8 + 8) of
// both heads (two 16-byte reads cover a 256-byte cache row per group), so a
// score is 16 FMAs per head plus a 3-level butterfly.  A round covers 32
// positions (8 warps x 4 groups); one online-softmax update absorbs two
// rounds.  The warps' states merge through shared memory.  With one split
// the output is written as the stacked bf16 hi/lo O-projection input (rows
// r and R + r, R = gridDim.y); with several, the CTA's unnormalized state
// (m0, l0, m1, l1, o0[128], o1[128]) goes to `partial` for merge_kernel.
constexpr int kAttRounds = 2;
constexpr int kAttTilePos = 32 * kAttRounds;            // positions per tile = one softmax update
constexpr int kAttTileBytes = kAttTilePos * kHeadDim * 2;  // K (or V) rows of one tile
constexpr int kAttStages = 3;
constexpr int kAttSmemBytes = kAttStages * 2 * kAttTileBytes;  // dynamic shared memory: 96 KB
constexpr unsigned long long kAttWaitNs = 1000000000ull;     // bound on one tile wait (1 s)
constexpr int kAttPartWords = 4 + 2 * kHeadDim;
constexpr int kAttMaxSplits = 16;
constexpr int kAttSplitRows = 64;  // splits > 1 only for up to this many rows

// Normalized attention output of dims d..d+3 of q head h, row r -> the
// stacked O-projection input (hi row r, lo row R + r).
__device__ __forceinline__ void store_att(__nv_bfloat16 *a2, int R, int r, int h, int d, const float (&y)[4]) {
  uint2 hi, lo;
  split4(y, hi, lo);
  *reinterpret_cast<uint2 *>(a2 + (size_t)r * kQSize + h * kHeadDim + d) = hi;
  *reinterpret_cast<uint2 *>(a2 + (size_t)(R + r) * kQSize + h * kHeadDim + d) = lo;
}

__global__ void __launch_bounds__(256) attention_kernel(
    const float *__restrict__ q, const __nv_bfloat16 *__restrict__ k_cache,
    const __nv_bfloat16 *__restrict__ v_cache, long long kv_seq_stride, int num_seqs, int layer, int max_seq_len,
    const int *__restrict__ row_seq, const int *__restrict__ row_pos, int splits, float *__restrict__ partial,
    __nv_bfloat16 *__restrict__ a2, unsigned *status) {
  pdl_wait();  // inputs are written by the previous kernel
  pdl_trigger();
  extern __shared__ __align__(128) uint8_t att_ring[];  // [stage][K tile | V tile]
  __shared__ __align__(16) float part[8 * kAttPartWords];
  __shared__ __align__(8) uint64_t full[kAttStages];
  const int g = blockIdx.x, r = blockIdx.y, sp = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = lane >> 3, r8 = lane & 7;
  const int seq = row_seq[r], pos = row_pos[r];
  const bool valid = seq >= 0 && seq < num_seqs && pos >= 0 && pos < max_seq_len;
  const int n = valid ? pos + 1 : 0;
  const int chunk = (n + splits - 1) / splits;
  const int j_lo = min(n, sp * chunk), j_hi = min(n, j_lo + chunk);
  float qv[2][16];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const float *qh = q + (size_t)r * kQSize + (2 * g + h) * kHeadDim;
    const float4 a = *reinterpret_cast<const float4 *>(qh + 8 * r8);
    const float4 b = *reinterpret_cast<const float4 *>(qh + 8 * r8 + 4);
    const float4 c = *reinterpret_cast<const float4 *>(qh + 64 + 8 * r8);
    const float4 d = *reinterpret_cast<const float4 *>(qh + 64 + 8 * r8 + 4);
    const float t[16] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w, c.x, c.y, c.z, c.w, d.x, d.y, d.z, d.w};
#pragma unroll
    for (int e = 0; e < 16; ++e) qv[h][e] = t[e];
  }
  const size_t head_off =
      (size_t)(valid ? seq : 0) * (size_t)kv_seq_stride + ((size_t)layer * kNumKVHeads + g) * (size_t)max_seq_len * kHeadDim;
  const uint8_t *kg = reinterpret_cast<const uint8_t *>(k_cache + head_off);
  const uint8_t *vg = reinterpret_cast<const uint8_t *>(v_cache + head_off);
  const int ntiles = (j_hi - j_lo + kAttTilePos - 1) / kAttTilePos;
  if (threadIdx.x == 0) {
#pragma unroll
    for (int st = 0; st < kAttStages; ++st) qmk::mbar_init(&full[st], 1);
    qmk::fence_mbar_init();
  }
  __syncthreads();
  // Tile t: positions [j_lo + 64 t, +n) into stage t % kAttStages (thread 0).
  const uint64_t pol = qmk::l2_policy_evict_first();
  auto issue = [&](int t) {
    if (t >= ntiles) return;
    const int st = t % kAttStages, j0 = j_lo + t * kAttTilePos;
    const unsigned bytes = (unsigned)(min(kAttTilePos, j_hi - j0) * kHeadDim * 2);
    uint8_t *dst = att_ring + (size_t)st * 2 * kAttTileBytes;
    qmk::mbar_arrive_expect_tx(&full[st], 2 * bytes);
    qmk::bulk_g2s(dst, kg + (size_t)j0 * (kHeadDim * 2), bytes, &full[st], pol);
    qmk::bulk_g2s(dst + kAttTileBytes, vg + (size_t)j0 * (kHeadDim * 2), bytes, &full[st], pol);
  };
  if (threadIdx.x == 0)
    for (int t = 0; t < kAttStages; ++t) issue(t);
  // Bounded wait for tile t (every thread); false after kAttWaitNs.
  auto wait_tile = [&](int t) -> bool {
    uint64_t *bar = &full[t % kAttStages];
    const unsigned par = (unsigned)(t / kAttStages) & 1u;
    uint64_t t0 = 0;
    for (unsigned it = 0;; ++it) {
      if (qmk::mbar_try_wait(bar, par)) return true;
      if ((it & 63u) == 63u) {
        const uint64_t now = qmk::global_timer_ns();
        if (t0 == 0) t0 = now;
        else if (now - t0 > kAttWaitNs) return false;
      }
    }
  };
  float mrun[2] = {-INFINITY, -INFINITY}, lrun[2] = {0.f, 0.f};
  float oacc[2][16];
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int e = 0; e < 16; ++e) oacc[h][e] = 0.f;

  int pending = ntiles;  // first tile not known to have landed
  for (int tile = 0; tile < ntiles; ++tile) {
    const int base = j_lo + tile * kAttTilePos;
    const bool landed = wait_tile(tile);
    const uint8_t *ks = att_ring + (size_t)(tile % kAttStages) * 2 * kAttTileBytes + 16 * r8;
    const uint8_t *vs = ks + kAttTileBytes;
    // warp-uniform: a warp with no position in this tile only joins the barrier
    if (landed && base + 4 * warp < j_hi) {
      int jr[kAttRounds];
      bool ok[kAttRounds];
      uint4 ka[kAttRounds], kb[kAttRounds], va[kAttRounds], vb[kAttRounds];
#pragma unroll
      for (int t = 0; t < kAttRounds; ++t) {
        const int j = 32 * t + 4 * warp + gq;  // row within the tile
        ok[t] = base + j < j_hi;
        jr[t] = ok[t] ? j : 4 * warp;  // an in-range row, masked below
        const uint8_t *kr = ks + jr[t] * (kHeadDim * 2);
        const uint8_t *vr = vs + jr[t] * (kHeadDim * 2);
        ka[t] = *reinterpret_cast<const uint4 *>(kr);
        kb[t] = *reinterpret_cast<const uint4 *>(kr + kHeadDim);
        va[t] = *reinterpret_cast<const uint4 *>(vr);
        vb[t] = *reinterpret_cast<const uint4 *>(vr + kHeadDim);
      }
      float s[kAttRounds][2];
#pragma unroll
      for (int t = 0; t < kAttRounds; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float *qq = qv[h];
          const unsigned w[8] = {ka[t].x, ka[t].y, ka[t].z, ka[t].w, kb[t].x, kb[t].y, kb[t].z, kb[t].w};
          float s0 = 0.f, s1 = 0.f;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            s0 = fmaf(qq[2 * k], bf_lo(w[k]), s0);
            s1 = fmaf(qq[2 * k + 1], bf_hi(w[k]), s1);
          }
          s[t][h] = s0 + s1;
        }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1)
#pragma unroll
        for (int t = 0; t < kAttRounds; ++t) {
          s[t][0] += __shfl_xor_sync(0xffffffffu, s[t][0], o);
          s[t][1] += __shfl_xor_sync(0xffffffffu, s[t][1], o);
        }
      float mn[2] = {mrun[0], mrun[1]};
#pragma unroll
      for (int t = 0; t < kAttRounds; ++t) {
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
        float pt[kAttRounds];
        float l = lrun[h] * corr;
#pragma unroll
        for (int t = 0; t < kAttRounds; ++t) {
          pt[t] = fast_exp2(s[t][h] - mn[h]);  // 0 for masked positions
          l += pt[t];
        }
        lrun[h] = l;
        mrun[h] = mn[h];
#pragma unroll
        for (int e = 0; e < 16; ++e) oacc[h][e] *= corr;
#pragma unroll
        for (int t = 0; t < kAttRounds; ++t) {
          const unsigned w[8] = {va[t].x, va[t].y, va[t].z, va[t].w, vb[t].x, vb[t].y, vb[t].z, vb[t].w};
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            oacc[h][2 * k] = fmaf(pt[t], bf_lo(w[k]), oacc[h][2 * k]);
            oacc[h][2 * k + 1] = fmaf(pt[t], bf_hi(w[k]), oacc[h][2 * k + 1]);
          }
        }
      }
    }
    // Stage tile % kAttStages fully read: refill it with tile + kAttStages.
    if (__syncthreads_or(!landed)) {
      if (threadIdx.x == 0 && status) atomicOr(status, QMK_BATCH_TIMEOUT);
      pending = tile;
      break;
    }
    if (threadIdx.x == 0) issue(tile + kAttStages);
  }
  // After a timeout: bounded wait for the copies still in flight before the
  // CTA (and its shared memory) goes away.
  // If that wait runs out too, copies may still be landing in this CTA's
  // shared memory after it exits: a status bit of its own says so.
  if (threadIdx.x == 0) {
    bool drained = true;
    for (int t = pending; t < ntiles && t < pending + kAttStages; ++t) drained = wait_tile(t) && drained;
    if (!drained && status) atomicOr(status, QMK_BATCH_COPIES_PENDING);
  }
  // Groups -> warp (same running max in every group): reduce-scatter, then
  // lane (gq, r8) holds head gq & 1, dims [base, base + 8), base = 8 r8 + 64 (gq >> 1).
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
  float *pw = part + warp * kAttPartWords;
  if (lane == 0) {
    pw[0] = mrun[0];
    pw[1] = lrun[0];
    pw[2] = mrun[1];
    pw[3] = lrun[1];
  }
  float4 *dst = reinterpret_cast<float4 *>(pw + 4 + (gq & 1) * kHeadDim + 64 * (gq >> 1) + 8 * r8);
  dst[0] = make_float4(fin[0], fin[1], fin[2], fin[3]);
  dst[1] = make_float4(fin[4], fin[5], fin[6], fin[7]);
  __syncthreads();
  // Thread i < 64: head i / 32, dims 4 (i % 32) .. + 3.
  if (threadIdx.x < 64) {
    const int hh = threadIdx.x >> 5, d = 4 * (threadIdx.x & 31);
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 8; ++w) M = fmaxf(M, part[w * kAttPartWords + 2 * hh]);
    float L = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const float mw = part[w * kAttPartWords + 2 * hh];
        if (mw != -INFINITY) {
          const float f = fast_exp2(mw - M);
          const float4 ow = *reinterpret_cast<const float4 *>(part + w * kAttPartWords + 4 + hh * kHeadDim + d);
          L += part[w * kAttPartWords + 2 * hh + 1] * f;
          o[0] += ow.x * f;
          o[1] += ow.y * f;
          o[2] += ow.z * f;
          o[3] += ow.w * f;
        }
      }
    }
    if (splits == 1) {
      const float inv = (L > 0.f) ? fast_rcp(L) : 0.f;
      const float y[4] = {o[0] * inv, o[1] * inv, o[2] * inv, o[3] * inv};
      store_att(a2, gridDim.y, r, 2 * g + hh, d, y);
    } else {
      float *pp = partial + (((size_t)r * kNumKVHeads + g) * splits + sp) * kAttPartWords;
      if ((threadIdx.x & 31) == 0) {
        pp[2 * hh] = M;
        pp[2 * hh + 1] = L;
      }
      *reinterpret_cast<float4 *>(pp + 4 + hh * kHeadDim + d) = make_float4(o[0], o[1], o[2], o[3]);
    }
  }
}

// Merge of the split states of (row r, KV head g): grid (g, r), 64 threads,
// thread i: q head 2g + i / 32, dims 4 (i % 32) .. + 3.
__global__ void __launch_bounds__(64) merge_kernel(const float *__restrict__ partial, int splits,
                                                   __nv_bfloat16 *__restrict__ a2) {
  pdl_wait();  // inputs are written by the previous kernel
  pdl_trigger();
  const int g = blockIdx.x, r = blockIdx.y;
  const int hh = threadIdx.x >> 5, d = 4 * (threadIdx.x & 31);
  const float *pp = partial + ((size_t)r * kNumKVHeads + g) * splits * kAttPartWords;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, pp[s * kAttPartWords + 2 * hh]);
  float L = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
  if (M != -INFINITY) {
    for (int s = 0; s < splits; ++s) {
      const float ms = pp[s * kAttPartWords + 2 * hh];
      if (ms != -INFINITY) {
        const float f = fast_exp2(ms - M);
        const float4 os = *reinterpret_cast<const float4 *>(pp + s * kAttPartWords + 4 + hh * kHeadDim + d);
        L += pp[s * kAttPartWords + 2 * hh + 1] * f;
        o[0] += os.x * f;
        o[1] += os.y * f;
        o[2] += os.z * f;
        o[3] += os.w * f;
      }
    }
  }
  const float inv = (L > 0.f) ? fast_rcp(L) : 0.f;
  const float y[4] = {o[0] * inv, o[1] * inv, o[2] * inv, o[3] * inv};
  store_att(a2, gridDim.y, r, 2 * g + hh, d, y);
}

// Prompt attention on the tensor cores (QmkBatchArgs.causal_run: the rows
// are positions 0 .. R-1 of sequence 0).  Per KV head g the two q heads'
// rows are stacked with their bf16 hi/lo halves, qs_g = [q_2g hi; q_2g+1 hi;
// q_2g lo; q_2g+1 lo] (4R x 128), so scores = qs_g K_g^T and out = P_g V_g
// are two batched GEMMs over the 8 heads (cuBLAS, fp32 accumulate) reading
// the cache in place; between them one kernel adds the hi/lo score rows,
// applies the causal mask and the softmax (exp2: q carries log2 e) and
// writes P as a stacked bf16 hi/lo pair.
constexpr int kGemmAttnMaxRows = 2048;

// qs[g][hh R + r] (hi) and qs[g][2R + hh R + r] (lo) <- q[r][(2g + hh) 128 + :]
__global__ void __launch_bounds__(256) qsplit_kernel(const float *__restrict__ q, __nv_bfloat16 *__restrict__ qs) {
  pdl_wait();  // inputs are written by the previous kernel
  pdl_trigger();
  const int r = blockIdx.x, R = gridDim.x;
  const int c = 8 * threadIdx.x;  // 8 of the row's 2048 values
  const int h = c >> 7, d = c & 127, g = h >> 1, hh = h & 1;
  const float4 a = *reinterpret_cast<const float4 *>(q + (size_t)r * kQSize + c);
  const float4 b = *reinterpret_cast<const float4 *>(q + (size_t)r * kQSize + c + 4);
  const float va[4] = {a.x, a.y, a.z, a.w}, vb[4] = {b.x, b.y, b.z, b.w};
  uint2 h0, l0, h1, l1;
  split4(va, h0, l0);
  split4(vb, h1, l1);
  __nv_bfloat16 *hi = qs + ((size_t)g * 4 * R + (size_t)hh * R + r) * kHeadDim + d;
  __nv_bfloat16 *lo = qs + ((size_t)g * 4 * R + 2 * (size_t)R + (size_t)hh * R + r) * kHeadDim + d;
  *reinterpret_cast<uint4 *>(hi) = make_uint4(h0.x, h0.y, h1.x, h1.y);
  *reinterpret_cast<uint4 *>(lo) = make_uint4(l0.x, l0.y, l1.x, l1.y);
}

// Softmax of score row i (< 2R: q head 2g + i / R, position r = i % R) over
// keys j <= r: s_j = S[g][i][j] + S[g][2R + i][j]; P[g][i][j] / P[g][2R+i][j]
// = bf16 hi / lo of exp2(s_j - max) / sum, zero for j > r (P rows at a
// stride of Rp >= R elements, a multiple of 8 for the GEMM's TMA).  Grid (2R, 8),
// 256 threads, up to kGemmAttnMaxRows / 256 keys per thread.
__global__ void __launch_bounds__(256) softmax_split_kernel(const float *__restrict__ S,
                                                            __nv_bfloat16 *__restrict__ P, int R, int Rp) {
  pdl_wait();  // inputs are written by the previous kernel
  pdl_trigger();
  __shared__ float red[8];
  constexpr int kPer = kGemmAttnMaxRows / 256;
  const int i = blockIdx.x, g = blockIdx.y, r = i % R;
  const float *s_hi = S + ((size_t)g * 4 * R + i) * R;
  const float *s_lo = S + ((size_t)g * 4 * R + 2 * (size_t)R + i) * R;
  float v[kPer];
  float m = -INFINITY;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int j = threadIdx.x + 256 * k;
    v[k] = (j <= r) ? s_hi[j] + s_lo[j] : -INFINITY;
    m = fmaxf(m, v[k]);
  }
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  m = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w]);
  float l = 0.f;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    v[k] = (v[k] == -INFINITY) ? 0.f : fast_exp2(v[k] - m);
    l += v[k];
  }
  const float inv = 1.f / block_sum256(l, red);  // key 0 is always present: sum >= 1
  __nv_bfloat16 *p_hi = P + ((size_t)g * 4 * R + i) * Rp;
  __nv_bfloat16 *p_lo = P + ((size_t)g * 4 * R + 2 * (size_t)R + i) * Rp;
  // The P V GEMM (causal mode 2, query tiles of at most 128 rows) reads row
  // r's keys only up to the end of its query tile; with R a multiple of 128
  // no tile spans two heads' rows, so keys past r's 128-aligned block are
  // never read and are not written.
  const int jend = (R % 128 == 0) ? min(R, (r / 128 + 1) * 128) : R;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int j = threadIdx.x + 256 * k;
    if (j < jend) {
      const float pv = v[k] * inv;
      const __nv_bfloat16 hb = __float2bfloat16(pv);
      p_hi[j] = hb;
      p_lo[j] = __float2bfloat16(pv - __bfloat162float(hb));
    }
  }
}

// att[r][(2g + hh) 128 + d] = O[g][hh R + r][d] + O[g][2R + hh R + r][d] -> the
// stacked O-projection input.  Grid: rows, 256 threads, 8 values each.
__global__ void __launch_bounds__(256) att_combine_kernel(const float *__restrict__ Ob, __nv_bfloat16 *__restrict__ a2) {
  pdl_wait();  // inputs are written by the previous kernel
  pdl_trigger();
  const int r = blockIdx.x, R = gridDim.x;
  const int c = 8 * threadIdx.x;
  const int h = c >> 7, d = c & 127, g = h >> 1, hh = h & 1;
  const float *hi = Ob + ((size_t)g * 4 * R + (size_t)hh * R + r) * kHeadDim + d;
  const float *lo = Ob + ((size_t)g * 4 * R + 2 * (size_t)R + (size_t)hh * R + r) * kHeadDim + d;
#pragma unroll
  for (int k = 0; k < 8; k += 4) {
    const float4 x = *reinterpret_cast<const float4 *>(hi + k), y = *reinterpret_cast<const float4 *>(lo + k);
    const float s4[4] = {x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w};
    store_att(a2, R, r, h, d + k, s4);
  }
}

// Vt[g][d][p] = V[g][p][d] for positions p < R of one layer's V cache (the
// P V GEMM wants both operands K-major: K = positions).  Grid (ceil(R / 64),
// 8 KV heads), 256 threads; a 64-position x 128-dim tile through shared
// memory.  Vt rows at a stride of Rp elements.
__global__ void __launch_bounds__(256) vtrans_kernel(const __nv_bfloat16 *__restrict__ v_layer, long long head_stride,
                                                     int R, int Rp, __nv_bfloat16 *__restrict__ vt) {
  pdl_wait();  // inputs are written by the previous kernel
  pdl_trigger();
  __shared__ __nv_bfloat16 t[64][kHeadDim + 2];
  const int p0 = blockIdx.x * 64, g = blockIdx.y;
  const __nv_bfloat16 *src = v_layer + (size_t)g * (size_t)head_stride;
  for (int i = threadIdx.x; i < 64 * kHeadDim; i += 256) {
    const int p = i / kHeadDim, d = i % kHeadDim;
    t[p][d] = (p0 + p < R) ? src[(size_t)(p0 + p) * kHeadDim + d] : __float2bfloat16(0.f);
  }
  __syncthreads();
  __nv_bfloat16 *dst = vt + (size_t)g * kHeadDim * (size_t)Rp;
  for (int i = threadIdx.x; i < 64 * kHeadDim; i += 256) {
    const int d = i / 64, p = i % 64;
    if (p0 + p < R) dst[(size_t)d * Rp + p0 + p] = t[p][d];
  }
}

// m = SiLU(gate) * up from the stacked gate|up GEMM output gu2 [2R, 6144]
// (nsplit K-split partials split_stride floats apart), split into the stacked down-projection input a2 [2R, 3072].  Grid: rows
// (R = gridDim.x), 256 threads, 12 elements each.
__global__ void __launch_bounds__(256) silu_split_kernel(const float *__restrict__ gu2,
                                                         __nv_bfloat16 *__restrict__ a2, int nsplit,
                                                         long long split_stride) {
  pdl_wait();  // inputs are written by the previous kernel
  pdl_trigger();
  const int r = blockIdx.x, R = gridDim.x;
  for (int c = threadIdx.x; c < kInter / 4; c += 256) {
    float gg[4] = {0.f, 0.f, 0.f, 0.f}, uu[4] = {0.f, 0.f, 0.f, 0.f};
    for (int sp = 0; sp < nsplit; ++sp) {  // K-split partials in split order
      const float *hi_row = gu2 + (size_t)sp * (size_t)split_stride + (size_t)r * (2 * kInter);
      const float *lo_row = gu2 + (size_t)sp * (size_t)split_stride + (size_t)(R + r) * (2 * kInter);
      const float4 gh = reinterpret_cast<const float4 *>(hi_row)[c], gl = reinterpret_cast<const float4 *>(lo_row)[c];
      const float4 uh = reinterpret_cast<const float4 *>(hi_row + kInter)[c];
      const float4 ul = reinterpret_cast<const float4 *>(lo_row + kInter)[c];
      gg[0] += gh.x + gl.x; gg[1] += gh.y + gl.y; gg[2] += gh.z + gl.z; gg[3] += gh.w + gl.w;
      uu[0] += uh.x + ul.x; uu[1] += uh.y + ul.y; uu[2] += uh.z + ul.z; uu[3] += uh.w + ul.w;
    }
    float y[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) y[e] = gg[e] * fast_rcp(1.0f + fast_exp2(-gg[e] * kLog2e)) * uu[e];
    uint2 h, l;
    split4(y, h, l);
    reinterpret_cast<uint2 *>(a2 + (size_t)r * kInter)[c] = h;
    reinterpret_cast<uint2 *>(a2 + (size_t)(R + r) * kInter)[c] = l;
  }
}

// Logits of output row i = row i + row O + i of the stacked LM-head GEMM
// output (O = gridDim.x), written to `logits` if given; greedy token:
// largest value, lowest index on ties.  1024 threads.
__global__ void __launch_bounds__(1024) argmax_kernel(const float *__restrict__ logits2, float *__restrict__ logits,
                                                      int *__restrict__ out) {
  pdl_wait();  // inputs are written by the previous kernel
  pdl_trigger();
  __shared__ float sv[32];
  __shared__ int si[32];
  const int i = blockIdx.x, O = gridDim.x;
  const float *hi = logits2 + (size_t)i * kVocab;
  const float *lo = logits2 + (size_t)(O + i) * kVocab;
  float *dst = logits ? logits + (size_t)i * kVocab : nullptr;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int c = threadIdx.x; c < kVocab; c += 1024) {
    const float v = hi[c] + lo[c];
    if (dst) dst[c] = v;
    if (v > best) {  // c increases per thread: strict > keeps the lowest index
      best = v;
      bi = c;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    best = sv[threadIdx.x];
    bi = si[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (threadIdx.x == 0 && out) out[i] = (bi == 0x7fffffff) ? 0 : bi;
  }
}

}  // namespace qmb

// =============================================================================
// Host side
// =============================================================================
namespace {

int fail(int code, const char *fmt, ...) {
  char msg[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(msg, sizeof(msg), fmt, ap);
  va_end(ap);
  return qmk_internal_set_error(code, msg);
}

constexpr size_t kAlign = 256;

size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

// Workspace regions for R rows and O output rows, in order (GEMM inputs and
// outputs stacked: 2R or 2O rows, hi halves then lo halves).
struct Layout {
  size_t x, a2, qkv2, q, c2, gu2, partial, qs, sc, pr, vt, ob, lm2, logits2, total;
};

// K splits of a projection GEMM with n outputs over rows2 stacked rows: with
// few rows the GEMM has few 128 x TN tiles (n / 128 weight-row tiles, one
// activation tile), too few CTAs to stream the weights at HBM speed; K
// chunks multiply the CTAs (up to ~one wave of 148 SMs) and the consumer of
// the output adds the partial products in split order.
constexpr int kMaxSplitK = 8;
int gemm_tile_n(int rows2) { return rows2 <= 32 ? 32 : rows2 <= 64 ? 64 : rows2 <= 128 ? 128 : 64; }  // activation tile of qmk_internal_gemm
int split_k(int n, int rows2, int k) {
  const int tiles = ((n + 127) / 128) * ((rows2 + gemm_tile_n(rows2) - 1) / gemm_tile_n(rows2));
  int s = 1;
  while (2 * s <= kMaxSplitK && 2 * s * tiles <= 148 && k / (2 * s) >= 256) s *= 2;
  return s;
}
// Rows of a split-K output region for up to R rows: max over r <= R of
// splits(r) 2r (so that a workspace for R rows serves every smaller call).
size_t split_rows(int R, int n, int k) {
  size_t best = 0;
  for (int r = 1; r <= R; ++r) {
    const size_t v = (size_t)split_k(n, 2 * r, k) * 2 * (size_t)r;
    if (v > best) best = v;
  }
  return best;
}
int round8(int v) { return (v + 7) / 8 * 8; }

Layout layout(int R, int O) {
  using namespace qmb;
  Layout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align_up(off + bytes);
    return at;
  };
  L.x = take((size_t)R * kHidden * 4);
  L.a2 = take((size_t)2 * R * kInter * 2);  // largest GEMM input: K = 3072
  L.qkv2 = take(split_rows(R, kQKV, kHidden) * kQKV * 4);
  L.q = take((size_t)R * kQSize * 4);
  L.c2 = take(std::max(split_rows(R, kHidden, kQSize), split_rows(R, kHidden, kInter)) * kHidden * 4);
  L.gu2 = take(split_rows(R, 2 * kInter, kHidden) * 2 * kInter * 4);
  // split states (used up to kAttSplitRows rows; sized so that the total
  // grows with R: a workspace for R rows serves every smaller call)
  L.partial = take((size_t)(R < kAttSplitRows ? R : kAttSplitRows) * kNumKVHeads * kAttMaxSplits * kAttPartWords * 4);
  // tensor-core prompt attention (causal runs of kAttSplitRows < R rows;
  // sized for min(R, kGemmAttnMaxRows) so that the total grows with R)
  const size_t Rg = (R > kAttSplitRows) ? (size_t)(R < kGemmAttnMaxRows ? R : kGemmAttnMaxRows) : 0;
  const size_t Rgp = (size_t)round8((int)Rg);
  L.qs = take(kNumKVHeads * 4 * Rg * kHeadDim * 2);
  L.sc = take(kNumKVHeads * 4 * Rg * Rg * 4);
  L.pr = take(kNumKVHeads * 4 * Rg * Rgp * 2);
  L.vt = take(kNumKVHeads * kHeadDim * Rgp * 2);
  L.ob = take(kNumKVHeads * 4 * Rg * kHeadDim * 4);
  L.lm2 = take((size_t)2 * O * kHidden * 2);
  L.logits2 = take((size_t)2 * O * kVocab * 4);
  L.total = off;
  return L;
}

// Position splits of the attention for R rows: as many CTAs (8 R splits) as
// fit resident at once (2 per SM on 148 SMs: one wave, no tail) when the
// batch is small, one split otherwise.
int attention_splits(int R) {
  using namespace qmb;
  if (R > kAttSplitRows) return 1;
  const int s = (2 * 148) / (kNumKVHeads * R);
  return s < 1 ? 1 : (s > kAttMaxSplits ? kAttMaxSplits : s);
}

// Every kernel of the forward pass is launched with programmatic stream
// serialization: it may be scheduled while its predecessor still runs and
// waits (pdl_wait) before touching the predecessor's data, so launch latency
// and prologues overlap the previous kernel; the GEMM prefetches its weight
// tiles before that wait.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

constexpr int kMaxDevices = 64;
bool g_att_smem_set[kMaxDevices] = {};  // attention_kernel's dynamic shared memory limit raised
std::mutex g_batch_mutex;

}  // namespace

__attribute__((visibility("hidden"))) int qmk_internal_gemm(
    const void *W, long long ldw, long long w_batch_stride, int n, const void *A, long long lda,
    long long a_batch_stride, int rows, int k, int batch, int splits, float *C, long long ldc, long long c_batch_stride,
    long long c_split_stride, unsigned *status, cudaStream_t stream, int causal, int causal_R, int w_static);

extern "C" size_t qmk_batch_workspace_bytes(int num_rows, int num_out) {
  if (num_rows < 1 || num_rows > QMK_BATCH_MAX_ROWS || num_out < 0 || num_out > num_rows) return 0;
  return layout(num_rows, num_out).total;
}

extern "C" int qmk_batch_forward(const QmkBatchArgs *a, cudaStream_t stream) {
  using namespace qmb;
  qmk_internal_clear_error();
  if (!a) return fail(QMK_ERR_ARGS, "qmk_batch_forward: null args");
  if (!a->embed_weight || !a->layer_ptrs || !a->final_norm_weight || !a->lm_head_weight || !a->cos_table ||
      !a->sin_table || !a->k_cache || !a->v_cache || !a->tokens || !a->row_seq || !a->row_pos)
    return fail(QMK_ERR_ARGS, "qmk_batch_forward: null weight/table/cache/row pointer");
  if (a->num_rows < 1 || a->num_rows > QMK_BATCH_MAX_ROWS)
    return fail(QMK_ERR_ARGS, "qmk_batch_forward: num_rows=%d outside [1, %d]", a->num_rows, QMK_BATCH_MAX_ROWS);
  if (a->num_out < 0 || a->num_out > a->num_rows)
    return fail(QMK_ERR_ARGS, "qmk_batch_forward: num_out=%d outside [0, num_rows=%d]", a->num_out, a->num_rows);
  if (a->num_out > 0 && !a->out_rows) return fail(QMK_ERR_ARGS, "qmk_batch_forward: num_out > 0 needs out_rows");
  if (a->num_layers < 1 || a->num_layers > QMK_MAX_LAYERS)
    return fail(QMK_ERR_ARGS, "qmk_batch_forward: num_layers=%d outside [1, %d]", a->num_layers, QMK_MAX_LAYERS);
  if (a->max_seq_len < 1 || a->num_seqs < 1)
    return fail(QMK_ERR_ARGS, "qmk_batch_forward: max_seq_len=%d num_seqs=%d", a->max_seq_len, a->num_seqs);
  const long long per_seq = (long long)a->num_layers * kNumKVHeads * a->max_seq_len * kHeadDim;
  if (a->num_seqs > 1 && a->kv_seq_stride < per_seq)
    return fail(QMK_ERR_ARGS, "qmk_batch_forward: kv_seq_stride=%lld < one cache (%lld elements)", a->kv_seq_stride,
                per_seq);
  // The attention copies cache rows with 1-D bulk copies: 16-byte aligned
  // sources (cache bases and the per-sequence stride).
  if ((reinterpret_cast<uintptr_t>(a->k_cache) | reinterpret_cast<uintptr_t>(a->v_cache)) % 16)
    return fail(QMK_ERR_ARGS, "qmk_batch_forward: k_cache / v_cache not 16-byte aligned");
  if (a->num_seqs > 1 && a->kv_seq_stride % 8)
    return fail(QMK_ERR_ARGS, "qmk_batch_forward: kv_seq_stride=%lld not a multiple of 8 elements (16 bytes)",
                a->kv_seq_stride);
  for (int i = 0; i < a->num_layers * 11; ++i)
    if (!a->layer_ptrs[i]) return fail(QMK_ERR_ARGS, "qmk_batch_forward: layer pointer %d is null", i);
  const Layout Lw = layout(a->num_rows, a->num_out);
  if (!a->workspace || a->workspace_bytes < Lw.total || (reinterpret_cast<uintptr_t>(a->workspace) % kAlign))
    return fail(QMK_ERR_WORKSPACE, "qmk_batch_forward: workspace needs %zu bytes, 256-byte aligned", Lw.total);

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(QMK_ERR_CUDA, "qmk_batch_forward: cudaGetDevice: %s", cudaGetErrorString(e));

  std::lock_guard<std::mutex> lock(g_batch_mutex);
  if (!g_att_smem_set[dev]) {
    e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttSmemBytes);
    if (e != cudaSuccess) return fail(QMK_ERR_CUDA, "attention_kernel shared memory: %s", cudaGetErrorString(e));
    g_att_smem_set[dev] = true;
  }
  uint8_t *ws = static_cast<uint8_t *>(a->workspace);

  const int R = a->num_rows, O = a->num_out, R2 = 2 * R;
  float *x = reinterpret_cast<float *>(ws + Lw.x);
  auto *a2 = reinterpret_cast<__nv_bfloat16 *>(ws + Lw.a2);
  float *qkv2 = reinterpret_cast<float *>(ws + Lw.qkv2);
  float *q = reinterpret_cast<float *>(ws + Lw.q);
  float *c2 = reinterpret_cast<float *>(ws + Lw.c2);
  float *gu2 = reinterpret_cast<float *>(ws + Lw.gu2);
  float *partial = reinterpret_cast<float *>(ws + Lw.partial);
  auto *qs = reinterpret_cast<__nv_bfloat16 *>(ws + Lw.qs);
  float *sc = reinterpret_cast<float *>(ws + Lw.sc);
  auto *pr = reinterpret_cast<__nv_bfloat16 *>(ws + Lw.pr);
  auto *vt = reinterpret_cast<__nv_bfloat16 *>(ws + Lw.vt);
  float *ob = reinterpret_cast<float *>(ws + Lw.ob);
  // causal run of a fresh prompt: attention as two tensor-core GEMMs per layer
  const bool gemm_attn = a->causal_run && R > kAttSplitRows && R <= kGemmAttnMaxRows;
  const int Rp = round8(R);  // row stride of P and Vt (16-byte aligned rows for the TMA)
  auto *lm2 = reinterpret_cast<__nv_bfloat16 *>(ws + Lw.lm2);
  float *logits2 = reinterpret_cast<float *>(ws + Lw.logits2);
  auto *kc = static_cast<__nv_bfloat16 *>(a->k_cache);
  auto *vc = static_cast<__nv_bfloat16 *>(a->v_cache);
  const auto *cos_t = static_cast<const __nv_bfloat16 *>(a->cos_table);
  const auto *sin_t = static_cast<const __nv_bfloat16 *>(a->sin_table);
  auto bf = [](const void *p) { return static_cast<const __nv_bfloat16 *>(p); };
  const int splits = attention_splits(R);
  const float *resid = nullptr;  // stacked output of the last down projection
  // K splits per projection (the same for O and down: n = 1024 both)
  const int s_qkv = split_k(kQKV, R2, kHidden), s_gu = split_k(2 * kInter, R2, kHidden);
  const int ks = split_k(kHidden, R2, kQSize);
  const long long qkv_stride = (long long)R2 * kQKV, gu_stride = (long long)R2 * 2 * kInter;
  const long long ks_stride = (long long)R2 * kHidden;  // floats between K-split partials
  static_assert(kQSize % (64 * kMaxSplitK) == 0 && kInter % (64 * kMaxSplitK) == 0 &&
                    kHidden % (64 * kMaxSplitK) == 0,
                "K chunks must stay whole 64-element blocks");
  unsigned *st = a->status;
  // C[rows, n] (+ nsplit partials) = A[rows, k] W[n, k]^T, row-major operands
  auto gemm = [&](int rows, int n, int k, const void *W, const void *A, float *C, int ldc, int nsplit,
                  long long split_stride) {
    // model weights: independent of the previous kernel (prefetched early)
    return qmk_internal_gemm(W, k, 0, n, A, k, 0, rows, k, 1, nsplit, C, ldc, 0, split_stride, st, stream, 0, 0, 1);
  };
  int rc = QMK_OK;

  launch_pdl(embed_kernel, dim3(R), dim3(256), 0, stream, bf(a->embed_weight), a->tokens, x, a->status);
  for (int l = 0; l < a->num_layers && rc == QMK_OK; ++l) {
    const void *const *P = a->layer_ptrs + 11 * l;
    const void *const *F = a->fused_ptrs ? a->fused_ptrs + 2 * l : nullptr;
    launch_pdl(residual_norm_split_kernel, dim3(R), dim3(256), 0, stream, x, resid, nullptr, R, bf(P[0]), a2, ks, ks_stride);
    if (F) {
      rc = gemm(R2, kQKV, kHidden, F[0], a2, qkv2, kQKV, s_qkv, qkv_stride);
    } else {
      rc = gemm(R2, kQSize, kHidden, P[1], a2, qkv2, kQKV, s_qkv, qkv_stride);
      if (rc == QMK_OK) rc = gemm(R2, kKVSize, kHidden, P[2], a2, qkv2 + kQSize, kQKV, s_qkv, qkv_stride);
      if (rc == QMK_OK) rc = gemm(R2, kKVSize, kHidden, P[3], a2, qkv2 + kQSize + kKVSize, kQKV, s_qkv, qkv_stride);
    }
    if (rc != QMK_OK) break;
    launch_pdl(qk_rope_kv_kernel, dim3(R), dim3(256), 0, stream, qkv2, bf(P[4]), bf(P[5]), cos_t, sin_t, a->row_seq, a->row_pos, kc, vc,
                                            a->kv_seq_stride, a->num_seqs, l, a->max_seq_len,
                                            a->attn_scale * kLog2e, q, a->status, s_qkv, qkv_stride);
    if (gemm_attn) {
      // scores = qs K^T and out = P V per KV head, the cache read in place
      const long long head = (long long)a->max_seq_len * kHeadDim;  // elements between KV heads
      const __nv_bfloat16 *kl = kc + (size_t)l * kNumKVHeads * head, *vl = vc + (size_t)l * kNumKVHeads * head;
      launch_pdl(qsplit_kernel, dim3(R), dim3(256), 0, stream, q, qs);
      // (causal: key tiles after every query of a tile are skipped; the
      // softmax reads only keys j <= r)
      rc = qmk_internal_gemm(kl, kHeadDim, head, R, qs, kHeadDim, (long long)4 * R * kHeadDim, 4 * R, kHeadDim,
                             kNumKVHeads, 1, sc, R, (long long)4 * R * R, 0, st, stream, 1, R, 0);
      if (rc != QMK_OK) break;
      launch_pdl(softmax_split_kernel, dim3(dim3(2 * R, kNumKVHeads)), dim3(256), 0, stream, sc, pr, R, Rp);
      launch_pdl(vtrans_kernel, dim3(dim3((R + 63) / 64, kNumKVHeads)), dim3(256), 0, stream, vl, head, R, Rp, vt);
      // (causal: a query tile's K range ends at its last position; P is 0 beyond)
      rc = qmk_internal_gemm(vt, Rp, (long long)kHeadDim * Rp, kHeadDim, pr, Rp, (long long)4 * R * Rp, 4 * R, R,
                             kNumKVHeads, 1, ob, kHeadDim, (long long)4 * R * kHeadDim, 0, st, stream, 2, R, 0);
      if (rc != QMK_OK) break;
      launch_pdl(att_combine_kernel, dim3(R), dim3(256), 0, stream, ob, a2);
    } else {
      launch_pdl(attention_kernel, dim3(dim3(kNumKVHeads, R, splits)), dim3(256), kAttSmemBytes, stream, 
          q, kc, vc, a->kv_seq_stride, a->num_seqs, l, a->max_seq_len, a->row_seq, a->row_pos, splits, partial, a2,
          a->status);
      if (splits > 1) launch_pdl(merge_kernel, dim3(dim3(kNumKVHeads, R)), dim3(64), 0, stream, partial, splits, a2);
    }
    rc = gemm(R2, kHidden, kQSize, P[6], a2, c2, kHidden, ks, ks_stride);
    if (rc != QMK_OK) break;
    launch_pdl(residual_norm_split_kernel, dim3(R), dim3(256), 0, stream, x, c2, nullptr, R, bf(P[7]), a2, ks, ks_stride);  // x += O-proj
    if (F) {
      rc = gemm(R2, 2 * kInter, kHidden, F[1], a2, gu2, 2 * kInter, s_gu, gu_stride);
    } else {
      rc = gemm(R2, kInter, kHidden, P[8], a2, gu2, 2 * kInter, s_gu, gu_stride);
      if (rc == QMK_OK) rc = gemm(R2, kInter, kHidden, P[9], a2, gu2 + kInter, 2 * kInter, s_gu, gu_stride);
    }
    if (rc != QMK_OK) break;
    launch_pdl(silu_split_kernel, dim3(R), dim3(256), 0, stream, gu2, a2, s_gu, gu_stride);
    rc = gemm(R2, kHidden, kInter, P[10], a2, c2, kHidden, ks, ks_stride);
    resid = c2;  // added to x by the next norm
  }
  if (rc != QMK_OK) return rc;
  if (O > 0) {
    launch_pdl(residual_norm_split_kernel, dim3(O), dim3(256), 0, stream, x, resid, a->out_rows, R, bf(a->final_norm_weight), lm2, ks,
                                                      ks_stride);
    rc = gemm(2 * O, kVocab, kHidden, a->lm_head_weight, lm2, logits2, kVocab, 1, 0);
    if (rc != QMK_OK) return rc;
    launch_pdl(argmax_kernel, dim3(O), dim3(1024), 0, stream, logits2, a->logits, a->out_tokens);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(QMK_ERR_CUDA, "qmk_batch_forward launch: %s", cudaGetErrorString(e));
  return QMK_OK;
}
