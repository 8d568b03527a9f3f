// Static work partition of the decode megakernel, shared by host and device.
//
// One CTA per SM.  Every phase of a layer splits its output rows into
// contiguous per-CTA ranges; attention is split into (kv head, KV split)
// items; the split-KV partials are merged by 32 merge tasks (one per
// (q head, half of head_dim)).  Producer (TMA) and consumer warps walk the
// same ranges, so the tile stream they agree on is defined here once.
#pragma once

#ifdef __CUDACC__
#define QMK_HD __host__ __device__ __forceinline__
#else
#define QMK_HD inline
#endif

namespace qmk {

constexpr int kHidden = 1024;
constexpr int kInter = 3072;
constexpr int kNumQHeads = 16;
constexpr int kNumKVHeads = 8;
constexpr int kHeadDim = 128;
constexpr int kQSize = kNumQHeads * kHeadDim;    // 2048
constexpr int kKVSize = kNumKVHeads * kHeadDim;  // 1024
constexpr int kQKVRows = kQSize + 2 * kKVSize;   // 4096
constexpr int kVocab = 151936;
constexpr int kMaxLayers = 64;

constexpr int kMaxCtas = 160;
constexpr int kMinCtas = 64;
// Sequences of the batched instance (qmk_run_batch): every GEMV phase makes
// one pass over its weight tiles for all of them; attention items and merge
// tasks are per (sequence, ...).
constexpr int kBatchSeqs = 4;
constexpr int kMaxSeqs = kBatchSeqs;
constexpr int kMaxSplits = 18;
constexpr int kMergeTasks = 32;                     // 16 q heads x 2 halves
constexpr int kMergeDims = kHeadDim / 2;            // 64 dims per merge task
constexpr int kPartWords = 4 + 2 * kHeadDim;        // m0,l0,m1,l1,o0[128],o1[128]
constexpr int kMergeWordsPerSplit = 2 + kMergeDims; // m, l, o[64]

// Tile geometry of the shared-memory ring (all tiles <= kSlotBytes).
constexpr int kSlotBytes = 32768;
constexpr int kNumSlots = 6;
constexpr int kQKVTileRows = 16;   // 16 x 2 KB
constexpr int kOTileRows = 8;      //  8 x 4 KB
constexpr int kGUTileRows = 8;     //  8 x (2 KB gate + 2 KB up), interleaved
constexpr int kDTileRows = 4;      //  4 x 6 KB at an 8 KB pitch
constexpr int kDRowPitch = 8192;   // down rows in a tile: 3 segments of 2 KB + 2 KB unused
constexpr int kLMTileRows = 16;    // 16 x 2 KB
constexpr int kKVTilePos = 64;     // 64 x 256 B K + 64 x 256 B V
constexpr int kKVTileVOffset = kKVTilePos * kHeadDim * 2;  // 16 KB

struct Range {
  int begin;
  int end;
};

// Rows [c*n/N, (c+1)*n/N): balanced to within one row.  32-bit arithmetic
// (n * (ncta) <= 151936 * 160 < 2^31): a 64-bit division is a long software
// sequence on the GPU.
QMK_HD Range split_rows(int n, int cta, int ncta) {
  Range r;
  r.begin = (int)((unsigned)(n * cta) / (unsigned)ncta);
  r.end = (int)((unsigned)(n * (cta + 1)) / (unsigned)ncta);
  return r;
}

QMK_HD Range qkv_rows(int cta, int ncta) { return split_rows(kQKVRows, cta, ncta); }
QMK_HD Range o_rows(int cta, int ncta) { return split_rows(kHidden, cta, ncta); }
QMK_HD Range gu_rows(int cta, int ncta) { return split_rows(kInter, cta, ncta); }
QMK_HD Range d_rows(int cta, int ncta) { return split_rows(kHidden, cta, ncta); }
QMK_HD Range lm_rows(int cta, int ncta) { return split_rows(kVocab, cta, ncta); }

// Attention items: item i = (b * 8 + g) * splits + s (sequence b of nb) lives
// on CTA i.
QMK_HD int item_of_cta(int cta, int splits, int nb = 1) {
  return (cta < nb * kNumKVHeads * splits) ? cta : -1;
}

// Merge task j lives on CTA ncta-1-j: sequence j/32, q head (j%32)/2, dims
// [(j%2)*64, +64).
QMK_HD int merge_task_of_cta(int cta, int ncta, int nb = 1) {
  int j = ncta - 1 - cta;
  return (j >= 0 && j < nb * kMergeTasks) ? j : -1;
}

// Previous positions [0, prev) of a KV head are cut into `splits` chunks.
QMK_HD Range kv_chunk(int prev, int s, int splits) {
  Range r;
  if (prev <= (1 << 26)) {  // prev * (s + 1) <= 2^26 * kMaxSplits < 2^31: 32-bit division
    r.begin = (int)((unsigned)(prev * s) / (unsigned)splits);
    r.end = (int)((unsigned)(prev * (s + 1)) / (unsigned)splits);
  } else {
    r.begin = (int)(((long long)prev * s) / splits);
    r.end = (int)(((long long)prev * (s + 1)) / splits);
  }
  return r;
}

// Splits per KV head for a launch whose largest "previous positions" count is
// max_prev: ~64 positions per split, at most kMaxSplits and at most ncta/8.
QMK_HD int attention_splits(int ncta, int max_prev, int nb = 1) {
  int s = (max_prev + 63) / 64;
  int cap = ncta / (kNumKVHeads * nb);
  if (cap > kMaxSplits) cap = kMaxSplits;
  if (s > cap) s = cap;
  if (s < 1) s = 1;
  return s;
}

// Workspace layout (bytes).  Control block first, then the 8-byte dataflow
// ("LL": value | flag << 32) buffers.
// Per-sequence buffers are kMaxSeqs consecutive copies (sequence b at b x
// the per-sequence size).
constexpr int kCtrlBytes = 16384;
constexpr int kWordsX = kHidden;
constexpr int kWordsQKV = kQKVRows;
constexpr int kWordsPart = kMaxCtas * kPartWords;  // one PART record per attention item (<= one per CTA)
constexpr int kWordsAtt = kQSize;
constexpr int kWordsA = kHidden;
constexpr int kWordsM = kInter;
constexpr int kWordsArg = 2 * kMaxCtas;
constexpr int kMaxTopK = 64;                       // top-k sampling: candidate keys per CTA
constexpr int kWordsTopk = kMaxTopK * kMaxCtas;
constexpr long long kOffX = kCtrlBytes;
constexpr long long kOffQKV = kOffX + 8LL * kMaxSeqs * kWordsX;
constexpr long long kOffPart = kOffQKV + 8LL * kMaxSeqs * kWordsQKV;
constexpr long long kOffAtt = kOffPart + 8LL * kWordsPart;
constexpr long long kOffA = kOffAtt + 8LL * kMaxSeqs * kWordsAtt;
constexpr long long kOffM = kOffA + 8LL * kMaxSeqs * kWordsA;
constexpr long long kOffArg = kOffM + 8LL * kMaxSeqs * kWordsM;
constexpr long long kOffTopk = kOffArg + 8LL * kMaxSeqs * kWordsArg;
constexpr long long kOffLLEnd = kOffTopk + 8LL * kWordsTopk;  // end of the dataflow words
constexpr long long kWorkspaceBytes = (kOffLLEnd + 4095) / 4096 * 4096;

// Control block (first kCtrlBytes of the workspace).
struct Ctrl {
  unsigned epoch;       // flag epoch base for the next launch
  unsigned exit_count;  // CTAs that finished the current launch
  unsigned err_code;    // first device error of the current launch
  unsigned err_info;
  unsigned launches;
  unsigned pad[27];
  unsigned kv_ready[kMaxSeqs * kMaxLayers * kNumKVHeads];  // [seq][layer][kv head]: epoch of the last K/V row written
};
static_assert(sizeof(Ctrl) <= kCtrlBytes, "control block too large");

}  // namespace qmk
