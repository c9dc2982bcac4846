// Kernel-side argument structures shared by the host launcher and the kernels.
#pragma once
#include <stdint.h>

namespace oomattn {

constexpr int kHeadDim = 128;   // head_dim this library is built for (Qwen2.5 / Llama-3: 128)
constexpr int kPageSize = 16;   // tokens per KV page
constexpr int kMaxBatch = 128;  // sequence rows carried in one launch's parameters
constexpr int kMaxGroup = 8;    // q heads per kv head handled by one decode CTA
// Split-KV partials per (row, q head).  f32 caches: up to 64, a one-page split
// per CTA up to 1024 cached tokens (C1 f32 decode: 10.9 us at 33 splits, 12.3
// at 17).  bf16 caches keep 32: one row of 2048 tokens ran 2.8 us slower per
// layer step at 43 splits than at 26.
constexpr int kMaxSplits = 64;
constexpr int kMaxSplitsBf16 = 32;

// Per-launch sequence rows, passed by value so a launch needs no host->device
// metadata copy (and can be captured in a CUDA graph).
//   seq[i]: context sequence slot (selects the block-table row)
//   len[i]: cache slots visible to row i (decode) or the cache length before
//           the append (append kernels)
//   pos[i]: absolute RoPE position of the row's first new token (append)
struct SeqBatch {
  int n;
  int seq[kMaxBatch];
  int len[kMaxBatch];
  int pos[kMaxBatch];
};

// Paged KV pool of all layers: element (layer, page, kv, slot, d) lives at
// (((layer * n_pool_pages + page) * n_kv + kv) * kPageSize + slot) * kHeadDim + d.
// Page n_pool_pages - 1 is the null page: zero, never written, and the
// block-table entry of every unassigned logical page.
struct KVPool {
  void* k;
  void* v;
  const int* block_table;  // [max_seqs][max_pages_per_seq]
  int max_pages_per_seq;
  int n_pool_pages;        // including the null page
  int n_kv;
  int kv_bf16;
};

// Test-only launch flags of the decode kernel (DecodeArgs::test_flags).
enum : int {
  kTestDropDecodeCopies = 1,  // the bf16 producer issues no copies: every consumer wait runs out its limit
  kTestDropLinearCopies = 2,  // the Q8 tensor-core pass's producer issues no copies: its MMA and promoter waits run out
};

struct DecodeArgs {
  const float* q;       // [rows][n_heads][128], rotated
  float* out;           // (row, q head) output at out + ((row * n_heads) + head) * o_stride, 128 floats
  float* lse;           // natural log at lse[((row * n_heads) + head) * lse_stride]; may be null
  int o_stride;         // 128 for [rows][n_heads][128]; 132 for the packed (O, lse) layout
  int lse_stride;       // 1 for [rows][n_heads]; 132 for the packed layout
  int test_flags;       // 0 outside tests
  int layer;
  int n_heads;
  int group;            // n_heads / n_kv
  int max_splits;       // partial slots per (row, q head)
  float qscale;         // softmax scale * log2(e)
  float* part_o;        // [rows][n_heads][max_splits][128]
  float* part_lse;      // [rows][n_heads][max_splits], base 2
  unsigned* counters;   // [rows][n_kv], zero between launches
  int* status;
  unsigned long long timeout_ns;
};

// The split-KV decode grid as a list of work items, longest first: row slot r
// is row order[r], whose pages are split into nsplit[r] near-equal ranges
// (ceil(pages / nsplit) each) for every kv head; its items are
// [item0[r], item0[r + 1]), kv head major.
struct DecodeSched {
  int n;                      // row slots
  int order[kMaxBatch];
  int nsplit[kMaxBatch];
  int item0[kMaxBatch + 1];
};

struct AppendArgs {
  const void* q;        // [T][n_heads][128]
  const void* k;        // [T][n_kv][128]
  const void* v;        // [T][n_kv][128]
  int in_bf16;
  void* q_out;          // [T][n_heads][128]
  int q_out_bf16;
  const float* bq;      // optional biases, added before RoPE
  const float* bk;
  const float* bv;
  const float* cos_t;   // [max_pos][64]
  const float* sin_t;
  int max_pos;
  int n_heads;
  int n_new;            // tokens per row; token t belongs to row t / n_new
  int layer;
  int variant;          // 0 split-half, 1 interleaved
  int rope_k;           // 0: store K as given (already rotated rows)
  int* status;
};

struct GemvArgs {
  const float* x;       // [T][hidden] f32
  const void* wq;       // [n_heads*128][hidden]
  const void* wk;       // [n_kv*128][hidden]
  const void* wv;
  int w_bf16;
  int hidden;
  int T;
  AppendArgs ap;        // epilogue (q/k/v pointers unused)
};

}  // namespace oomattn
