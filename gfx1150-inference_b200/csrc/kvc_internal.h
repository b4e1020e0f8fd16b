// Internal interface between the host runtime (kvc_host.cpp, kvc_offload.cpp)
// and the CUDA kernels (kvc_kernels.cu).  Not part of the public C ABI.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace kvc {

// Running-max sentinel for "no position seen yet".  Finite on purpose: the
// difference of two sentinels is 0, never NaN, and every weight that involves
// an empty partial is multiplied by a zero sum.
constexpr float kNegBig = -1.0e30f;
constexpr float kLog2e = 1.4426950408889634f;

// Upper bound of one mbarrier wait before a kernel gives up and reports
// KVC_DEVERR_WAIT_LIMIT (nanoseconds of %globaltimer).
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// Tokens per shared-memory slab.  A slab is the unit of one bulk copy per K and
// per V: 16 positions x head_dim of one KV head, contiguous in the pool for
// every layout and page size (page_size is a multiple of 16).
constexpr int kSlab = 16;

// ---- pool layouts -------------------------------------------------------------
// A page-head is one contiguous block of page_size x head_dim elements.  Inside
// it, positions and dims are arranged in 16-byte units (8 x 16-bit or 4 x fp32):
//   kLayoutCore   (16-bit storage): unit (t, u) at ((t / 8) * U + u) * 8 + t % 8,
//                 i.e. 8-position x 16-byte "core matrices" stored contiguously,
//                 the operand tile shape of ldmatrix / mma (and of tcgen05's
//                 no-swizzle canonical layout); reads are bank-conflict free.
//   kLayoutLinear (fp32 storage):  unit (t, u) at t * U + u, row-major.
// Both keep every 16-position slab contiguous, so a slab is one bulk copy.
enum : int { kLayoutCore = 0, kLayoutLinear = 1 };

__host__ __device__ __forceinline__ size_t unit_offset(int layout, int t, int u, int U) {
  return layout == kLayoutCore ? (static_cast<size_t>((t >> 3) * U + u) * 8 + (t & 7))
                               : (static_cast<size_t>(t) * U + u);
}


// Split-K chunk: every query's context is cut into splits of one length per
// batch (a multiple of the page size), 512 positions unless a single wave of
// shorter or longer splits is estimated faster (choose_split_tokens).  The
// partition depends only on the batch's context lengths and head counts, never
// on the storage mode, so resident and offloaded runs add in the same order.
constexpr int kSplitTokens = 512;
// Upper bound on pages per split the kernels accept (split tokens are capped at
// kMaxSplitPages * 16).
constexpr int kMaxSplitPages = 64;
// The persistent decode kernel runs kPersistWarpsPerSm independent warps per SM,
// as kPersistCtasPerSm CTAs of kPersistWarps warps.  Two 4-warp CTAs per SM
// rather than one 8-warp CTA: an SM takes the next launch's first CTA as soon as
// half of its warps are done, which measured 0.3-4 % faster per layer (most on
// the one-wave lists of the 8-way KV-head split) and never slower.
constexpr int kPersistWarps = 4;
constexpr int kPersistCtasPerSm = 2;
constexpr int kPersistWarpsPerSm = kPersistWarps * kPersistCtasPerSm;
// Slabs per warp brought into L2 while a decode launch waits for the preceding
// kernel (early KV streaming only), for plans whose queries all have the same
// context and whose splits are at least kL2AheadMinSplit positions long;
// KVC_L2_AHEAD overrides (0 ... 32).  Measured on B200 (replayed steps, A/B on
// one box): even contexts gain, one rank of config 4's 8-way and 2-way KV-head
// splits 2.3 % and 1.3 %, config 4 itself neutral; ragged batches lose, config 3's
// 2-way and 4-way shards 2.5 % and 1.3 % (growing loop 2-6 %), config 3 0.5 %;
// config 2's 112-position splits lose 7 %, hence the threshold; deeper prefetch
// was slower everywhere.
constexpr int kL2AheadSlabs = 2;
constexpr int kL2AheadMinSplit = 192;
// Ranks a head exchange can span (one process per GPU of one node).
constexpr int kMaxPeers = 8;

struct PoolGeom {
  int num_layers = 0;
  int num_pages = 0;
  int page_size = 0;
  int num_kv_heads = 0;
  int head_dim = 0;
  int dtype = 0;       // KVC_DTYPE_*
  int elem_size = 0;   // bytes per element
  int layout = 0;      // kLayoutCore / kLayoutLinear
  size_t page_head_bytes = 0;   // page_size * head_dim * elem_size
  size_t page_bytes = 0;        // num_kv_heads * page_head_bytes
  size_t layer_bytes = 0;       // num_pages * page_bytes
};

struct AppendArgs {
  uint8_t* k_layer;
  uint8_t* v_layer;
  const uint8_t* k_new;          // (n, Hkv, D) token-major rows
  const uint8_t* v_new;
  const int32_t* block_tables;   // (rows, bt_stride)
  const int32_t* rows;           // (n) block-table row per appended row, or null (row 0)
  const int32_t* positions;      // (n) position per appended row, or null (pos0 + i)
  int pos0;
  int bt_stride;
  int n;
  int num_kv_heads;
  int row_units;                 // head_dim * elem_size / 16
  int page_size;
  int num_pages;
  int layout;
  size_t page_head_bytes;
};

struct GatherArgs {
  const uint8_t* k_layer;
  const uint8_t* v_layer;
  uint8_t* k_out;                // (count, Hkv, D)
  uint8_t* v_out;
  const int32_t* bt_row;         // block-table row of the sequence
  int bt_stride;
  int start;
  int count;
  int num_kv_heads;
  int row_units;
  int page_size;
  int num_pages;
  int layout;
  size_t page_head_bytes;
};

// One split item: {query, split index, first position, end position}.
// One query record: {block-table row, context length, first split slot, splits}.
struct DecodeArgs {
  const uint8_t* k_layer;
  const uint8_t* v_layer;
  const void* q;                 // (n_queries, H, D)
  void* out;                     // (n_queries, H, D)
  const int32_t* block_tables;
  int bt_stride;
  const int4* items;             // 2 per item: {query, split, tb, te}, {row, ctx, slot0, splits}
  const int4* qinfo;
  float* part_o;                 // (split slots, H, D) fp32 partial outputs
  float2* part_ml;               // (split slots, H) running max (log2 units) and sum
  unsigned int* counters;        // (n_queries, Hkv, n_hchunk), zero between launches
  // Fused append (decode steps): when non-null, query i's new K/V row, (n_queries,
  // Hkv, D), is written at position ctx_i - 1 of its block-table row by the CTA
  // that owns that position, which also uses it in place of the slab's stale row.
  // Only valid when every query has its own block-table row.
  const uint8_t* k_new;
  const uint8_t* v_new;
  // Persistent schedule: n_units unit records, longest first, each 3 x int4:
  // {query, split, first pos, end pos}, {bt row, ctx, split slot0, n_splits},
  // {KV head, q-head chunk, first q-head, q-heads in chunk}.  Warp w of the grid
  // starts with unit w and takes further units from *queue (zero between
  // launches; the merge kernel re-arms it).
  const int4* sched_recs;
  int n_units;
  int sched_cap = 0;             // unit records sched_recs holds (>= n_units)
  unsigned int* queue;
  int n_sched_ctas;
  // Block tables and KV pages are not written by the kernel launched just before
  // (plan flag KVC_PLAN_KV_STABLE): the decode kernel may start streaming them
  // before that kernel's results are visible.
  int early_prefetch;
  int l2_ahead = 0;              // slabs per warp prefetched into L2 before the wait
  // queries with more than one split (merged by merge_splits_kernel)
  const int32_t* merge_queries;
  int n_merge_queries;
  int n_items;
  int num_heads;
  int num_kv_heads;
  int group;                     // num_heads / num_kv_heads
  int n_hchunk;                  // ceil(group / 8): q-head chunks per KV head
  int head_dim;
  int page_size;
  int num_pages;
  float scale_log2;              // scale * log2(e)
  int n_queries_total = 0;       // queries of the plan (merge grid of an exchange)
  int merge_wph = 1;             // merge warps per q-head: 1, 2, 4 or 8 (merge_warps_per_head)
  // Head exchange (KV heads split across GPUs): when xchg_peers > 0 every query's
  // output goes through the merge kernel, which stores each output row straight
  // into the exchange slot of all xchg_peers ranks (peer memory over NVLink) at
  // row stride out_heads * D and head offset out_head0; xchg_signal_kernel then
  // publishes the next epoch (epoch_ctr + 1) in this rank's flag word on every
  // rank (peer_flag[p] points at it) and waits until all ranks' flags show it.
  int xchg_peers = 0;
  int out_heads = 0;
  int out_head0 = 0;
  unsigned int* epoch_ctr = nullptr;       // this rank's last epoch (local, device-side)
  void* peer_out[kMaxPeers] = {};
  unsigned int* peer_flag[kMaxPeers] = {};
  const unsigned int* my_flags = nullptr;  // this rank's flag words, one per source rank
  unsigned long long wait_limit_ns = 0;
  // Host-buffer calls: device address of the page-locked copy of the device error
  // word, which the split merge (the last kernel of the call) stores, so the host
  // reads it after its wait without a copy of its own.  Null otherwise.
  uint32_t* err_host = nullptr;
  // Graph-stable plans (KVC_PLAN_GRAPH): the plan's device header, from which the
  // kernels read n_units, l2_ahead, the multi-split query count and the merge's
  // warps per head (kHdr*), so launches captured in a CUDA graph stay valid when
  // the plan is rebuilt for grown contexts.  The decode grid then spans every SM
  // and the merge grid n_queries x num_heads.  Null: the values above are used.
  const int* plan_hdr = nullptr;
};
// Slots of the plan's device header (int32).
constexpr int kHdrUnits = 0;
constexpr int kHdrL2Ahead = 1;
constexpr int kHdrMergeQueries = 2;
constexpr int kHdrMergeWph = 3;
constexpr int kHdrInts = 4;

struct FillArgs {
  uint8_t* base;                 // first byte of the range to fill
  size_t n_elems;
  uint64_t seed;
  uint64_t index0;               // global element index of base (for reproducibility)
  float stddev;
  int dtype;
};

// Warps of one split-merge CTA, and how many of them share one q-head (from the
// most splits of any query: about eight splits per warp, at most kMergeWarps
// warps).  8-warp CTAs rather than 16: a merge CTA then fits beside a decode CTA
// of the next launch (4 warps at 240 registers), 4 % faster per layer on one rank
// of the 8-way KV-head split of config 3 and within 0.4 % elsewhere.
constexpr int kMergeWarps = 8;
inline int merge_warps_per_head(int max_splits) {
  const int w = max_splits <= 8 ? 1 : max_splits <= 16 ? 2 : max_splits <= 32 ? 4 : 8;
  return w < kMergeWarps ? w : kMergeWarps;
}

// Copy of up to three host-mapped (page-locked) input buffers into device
// staging, 16 bytes per thread, by a kernel that lets the next launch (the
// decode, a programmatic dependent) start streaming KV while the copy runs.
// Every pointer is 16-byte aligned.
struct StageArgs {
  const uint8_t* src[3];
  uint8_t* dst[3];
  size_t bytes[3];
};

// Rotary position embedding of up to two tensors (q and the new K rows) of
// n_tokens tokens, (n_tokens, heads, D) each: the pair (i0, i1) of head h of
// token t is rotated by angle positions[t] * inv_freq[i] (positions == nullptr:
// pos0 + t), i0 = 2i, i1 = 2i + 1 (interleaved) or i0 = i, i1 = i + D/2 (NeoX),
// in fp32, rounded to the storage type (the rope kernel of rope.hip:21-55).
constexpr int kMaxRopePairs = 128;   // head_dim <= 256
struct RopeArgs {
  const uint8_t* src[2];
  uint8_t* dst[2];
  int heads[2];                      // 0: tensor absent
  int n_tokens;
  int head_dim;
  int dtype;
  int neox;
  int pos0;
  const int32_t* positions;
  float inv_freq[kMaxRopePairs];
};
// Host table inv_freq[i] = 1 / freq_base^(2i / head_dim) in fp32 (rope.hip:79-83).
void rope_inv_freq(float freq_base, int head_dim, float* out);

// Launchers: return cudaSuccess or the launch error.
cudaError_t launch_append(const AppendArgs& a, int elem_size, cudaStream_t s);
cudaError_t launch_gather(const GatherArgs& a, cudaStream_t s);
cudaError_t launch_stage_inputs(const StageArgs& a, cudaStream_t s);
// pdl: the rotation lets the next launch (a decode) start before it ends.
cudaError_t launch_rope(const RopeArgs& a, cudaStream_t s, bool pdl);
cudaError_t launch_fill_normal(const FillArgs& a, cudaStream_t s);
// kind: 0 = tensor-core kernel, 1 = CUDA-core kernel (selected by the host).
cudaError_t launch_decode(const DecodeArgs& a, int dtype, int layout, cudaStream_t s);
bool decode_uses_mma(int dtype, int head_dim, int page_size);

// Device error word (per device): read and optionally clear; its device address.
cudaError_t read_device_error(uint32_t* code, uint32_t* info, bool clear);
cudaError_t device_error_address(void** p);

// ---- layer pipeline (forward_layer_cached, attention.hip:603-695) ----------------
// Weight storage types: the GGML type ids forward_layer_cached takes
// (bindings.cpp:518-557).  Weights are (n, k) row-major, each row k / per blocks.
constexpr int kWF16 = 1, kWQ4_0 = 2, kWQ8_0 = 8, kWQ4_K = 12, kWQ6_K = 14;
// Weights per block and bytes per block of a type (0, 0 if unknown).
void weight_block(int w_type, int* per, int* bytes);

// y = x · Wᵀ for fp16 activations x (m, k) and quantized W (n, k); fp32 sums, fp16 y.
// Up to three matrices of one type and k in one launch (segments, e.g. q, k, v).
// Epilogues: kEpiStore (y), kEpiSwiglu (seg 0 = gate, seg 1 = up, same n:
// y = silu(gate) · up with both rounded to fp16 first, mlp.hip:18-31), kEpiResidual
// (y = res + fp16(x · Wᵀ), the second residual of attention.hip:689).
constexpr int kEpiStore = 0, kEpiSwiglu = 1, kEpiResidual = 2;
struct LinearSeg {
  const uint8_t* w = nullptr;
  __half* out = nullptr;
  int n = 0;        // rows of W = columns of y
  int out_ld = 0;   // elements between rows of y
};
struct LinearArgs {
  const __half* x = nullptr;
  int x_ld = 0;
  int m = 0, k = 0;
  int w_type = 0;
  size_t row_bytes = 0;
  LinearSeg seg[3];
  int n_seg = 0;
  int epi = kEpiStore;
  const __half* res = nullptr;   // kEpiResidual: (m, n) with ld seg[0].out_ld
  // set by the launcher
  int seg_cta0[4] = {0, 0, 0, 0};  // first CTA of each segment (prefix sums)
  int stages = 0;                  // staged kernel: ring depth
  uint32_t stage_row_bytes = 0;    // staged kernel: weight bytes of one row per stage
  int stage_tok = 0;               // staged kernel: token rows of x per stage (min(8·MT, m))
  uint32_t* err = nullptr;         // the device error word (bounded waits)
};
constexpr int kMaxLinStages = 16;
cudaError_t launch_linear(LinearArgs& a, cudaStream_t s);

// out = silu(gate) · up elementwise (gate and up of different weight types).
cudaError_t launch_swiglu(const __half* gate, const __half* up, __half* out, size_t n,
                          cudaStream_t s);

// RMSNorm of each row of x (m, k): x / sqrt(mean(x²) + eps) · w, fp16 out
// (rmsnorm.hip:23-74).  With res: h = fp16(x + res) is written to h_out and
// normalised instead (the fused residual + RMSNorm of rmsnorm.hip:79-140).
cudaError_t launch_rmsnorm(const __half* x, const __half* res, const __half* w, __half* h_out,
                           __half* out, int m, int k, float eps, cudaStream_t s);

}  // namespace kvc
