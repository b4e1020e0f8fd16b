// Host-side objects shared by kvc_host.cpp and kvc_offload.cpp.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <vector>

#include "kvc_internal.h"

namespace kvc {

// Grow-only device buffer.
struct DevBuf {
  void* ptr = nullptr;
  size_t cap = 0;
  cudaError_t ensure(size_t bytes);
  void release();
};

// Grow-only page-locked host buffer.
struct HostBuf {
  void* ptr = nullptr;
  size_t cap = 0;
  cudaError_t ensure(size_t bytes);
  void release();
};

int set_error(int code, const char* fmt, ...);
int cuda_error(cudaError_t e, const char* what);

// ---- host-side waits and fault injection ----
// Every wait of the host for the library's own GPU work polls (cudaStreamQuery /
// cudaEventQuery) against a wall-clock limit (kvc_set_host_wait_limit, 60 s by
// default) and returns KVC_ERR_TIMEOUT with `what` in the message when it runs out.
int wait_stream(cudaStream_t s, const char* what);
int wait_event(cudaEvent_t e, const char* what);
// kvc_test_inject_failure: true when this call at `site` (KVC_FAULT_*) is to fail.
bool injected_failure(int site);
// cudaMalloc / cudaHostAlloc / cudaHostRegister that honour kvc_test_inject_failure.
cudaError_t dev_alloc(void** p, size_t n);
cudaError_t host_alloc(void** p, size_t n, unsigned flags);
cudaError_t host_register(void* p, size_t n);
// cudaSetDevice with the library's status convention.
int use_device(int device);
int check_device_error(const char* what);
int elem_size_of(int dtype);
int make_geom(int num_layers, int num_pages, int page_size, int num_kv_heads, int head_dim,
              int dtype, PoolGeom* g);

}  // namespace kvc

// Paged KV pool: K and V each num_layers x num_pages x num_kv_heads page-heads.
struct kvc_pool {
  kvc::PoolGeom g;
  int device = 0;
  uint8_t* k = nullptr;
  uint8_t* v = nullptr;
  size_t cap_bytes = 0;   // bytes allocated per K (and per V), grow-only
  kvc::DevBuf io;         // staging for the host-buffer entry points
  kvc::HostBuf io_host;   // page-locked staging of pageable host buffers
};

// Split-K decode plan for one batch of queries.
struct kvc_plan {
  bool valid = false;
  int device = -1;
  int n_queries = 0, n_items = 0, n_slots = 0;
  int num_heads = 0, num_kv_heads = 0, group = 0, n_hchunk = 0;
  int head_dim = 0, page_size = 0, max_ctx = 0, max_splits = 0, split_tokens = 0;
  bool rows_distinct = true;   // every query has its own block-table row
  bool even_ctx = false;       // every query has the same context length
  int flags = 0;               // KVC_PLAN_*
  kvc::PoolGeom pool_geom;
  std::vector<int4> items, qinfo, item_pairs;
  std::vector<int32_t> rows, positions;
  std::vector<int4> sched_recs;   // 3 per scheduled unit
  std::vector<int32_t> merge_queries;
  int n_sched_ctas = 0, n_units = 0;
  int sms = 0;                  // SMs of the plan's device (its persistent grid's width)
  // Inputs of the last successful build (geometry, queries, contexts, rows): a
  // build with the same inputs keeps the uploaded plan (every layer of one
  // decode step plans the same queries).
  std::vector<int32_t> built_from;
  kvc::DevBuf d_blob;          // items, qinfo, rows, positions, unit records, merge list, counter
  kvc::DevBuf d_part_o, d_part_ml, d_counters;
  // device-error count when d_counters was last zeroed (a kernel that gave up
  // may leave split counters armed: a later build zeroes them again)
  uint32_t counters_zeroed_at = 0;
  // KVC_PLAN_GRAPH: capacities the blob and the split scratch are laid out for
  // (grow-only), the device addresses and launch shape captured launches hold,
  // and the generation that advances whenever a rebuild changes any of them.
  size_t cap_items = 0, cap_queries = 0, cap_sched = 0, cap_merge = 0, cap_slots = 0;
  std::vector<uintptr_t> launch_sig;
  uint64_t generation = 0;
  // parts of d_blob (set by the upload)
  const int4* dev_items = nullptr;
  const int4* dev_qinfo = nullptr;
  const int32_t* dev_rows = nullptr;
  const int32_t* dev_pos = nullptr;
  const int4* dev_sched = nullptr;
  const int32_t* dev_merge = nullptr;
  unsigned int* dev_queue = nullptr;
  const int* dev_hdr = nullptr;  // kHdr* counts (KVC_PLAN_GRAPH), next to the unit counter
  kvc::DevBuf d_rope;          // rotated q and new K rows (kvc_append_decode_rope)
  kvc::DevBuf d_layer;         // activations of kvc_forward_layer_paged
  kvc::HostBuf h_stage;
  cudaEvent_t upload_done = nullptr;

  void release() {
    d_blob.release();
    d_part_o.release();
    d_part_ml.release();
    d_counters.release();
    d_rope.release();
    d_layer.release();
    h_stage.release();
    if (upload_done) cudaEventDestroy(upload_done);
    upload_done = nullptr;
    built_from.clear();
    valid = false;
  }
};

// Head exchange between the ranks of one node (one process per GPU).  Device
// buffer (cudaMalloc, shared with the peers through CUDA IPC):
//   [0, 64)        flag words, one per source rank: the last epoch it published
//   [192, 196)     last epoch this rank published (local use only)
//   [256, ...)     n_slots output slots of slot_bytes each (256-byte aligned)
struct kvc_xchg {
  int device = 0, rank = 0, world = 1;
  size_t slot_bytes = 0, slot_stride = 0;
  int n_slots = 0;
  uint8_t* base = nullptr;                   // this rank's buffer
  uint8_t* peer_base[kvc::kMaxPeers] = {};   // every rank's buffer as mapped here
  bool ipc_opened[kvc::kMaxPeers] = {};      // mapped by kvc_xchg_connect (to close)
  bool connected = false;
  unsigned long long wait_limit_ns = 2000000000ull;
};

namespace kvc {
constexpr size_t kXchgFlagsOff = 0;
constexpr size_t kXchgEpochOff = 192;
constexpr size_t kXchgSlotsOff = 256;

// Where a decode's outputs go when KV heads are split across ranks.
struct XchgTarget {
  kvc_xchg* x;
  int slot;
  int out_heads;    // q-heads of the whole model (row stride of a slot)
  int out_head0;    // this rank's first q-head
};

// Device address of page-locked host memory (written directly by the kernels),
// or nullptr for pageable memory.
void* mapped_host_ptr(void* h);
// End of a host-buffer call on stream s: copy `bytes` of d_out to h_out unless
// the kernels wrote h_out directly (d_out == nullptr), read the device error
// word into page-locked memory on the same stream (unless `merged`: the split
// merge stored it there), wait for the stream, and report a device error under
// `what`.
int finish_host_call(cudaStream_t s, void* h_out, const void* d_out, size_t bytes,
                     const char* what, bool merged = false);
// Creates the page-locked copy of the device error word (once per device) before
// a host-buffer call launches its kernels; until finish_host_call, the decodes
// this thread launches store the word there (host_call_error_copy()).
int prepare_host_call();
uint32_t* host_call_error_copy();

// Host buffers of one host-buffer call (q, new K rows, new V rows; out).
// stage_host_call moves the inputs to d_in[] with the input staging kernel,
// which lets the decode behind it start streaming KV: page-locked inputs are
// read in place, pageable ones are first copied (on the CPU) into `pinned`.  It
// also picks where the kernels write the output: the host buffer itself when it
// is page-locked, else a page-locked block of `pinned` (*out_dev), which
// finish_staged_call copies to the host buffer after the wait.  The caller's
// previous call on the stream must have completed (every host-buffer call waits).
struct HostCallStage {
  void* out_dev = nullptr;      // where the kernels write the output
  void* out_bounce = nullptr;   // page-locked copy source after the wait (or null)
};
int stage_host_call(kvc::HostBuf& pinned, const void* const h_in[3], const size_t in_bytes[3],
                    uint8_t* const d_in[3], void* h_out, size_t out_bytes, cudaStream_t s,
                    HostCallStage* st);
// merged: the call's last kernel is the tensor-core decode's split merge, which
// keeps the error word's page-locked mirror current (no copy of its own needed).
int finish_staged_call(cudaStream_t s, void* h_out, const HostCallStage& st, size_t out_bytes,
                       const char* what, bool merged = false);

// Plans q_len queries at start_pos (row 0 of the block table) of a single
// sequence; run before any input staging so the plan's upload does not sit
// between the staging kernel and the attention kernel.
int cached_plan(kvc_pool* pool, kvc_plan* plan, int q_len, int start_pos, int num_heads,
                bool causal, cudaStream_t s);
// Appends the q_len rows and attends over the planned queries; early = 1 when the
// launch directly before writes no KV pages (input staging, RoPE).
int cached_run(kvc_pool* pool, const kvc_plan* plan, const int32_t* d_bt, int bt_len,
               const void* d_Q, const void* d_Kn, const void* d_Vn, void* d_Out, int layer_idx,
               int q_len, int start_pos, float scale, cudaStream_t s, int early);

// ---- layer pipeline (kvc_layer_host.cpp) ----
struct LayerDims {
  int layer = 0, seq = 0, pos = 0;
  int hidden = 0, inter = 0, H = 0, Hkv = 0, D = 0;
  float eps = 0.f, base = 0.f, scale = 0.f;
  bool neox = false;
};
// Device pointers of one layer; w / type in the order q, k, v, o, gate, up, down.
struct LayerIO {
  const __half* x_in = nullptr;
  __half* x_out = nullptr;
  const __half* attn_norm = nullptr;
  const __half* ffn_norm = nullptr;
  const void* w[7] = {};
  int type[7] = {};
};
int check_weight(int w_type, int n, int k, const char* name);
size_t weight_size(int w_type, int n, int k);
int check_layer(const LayerDims& d, const int* types);
// Total bytes (256-byte aligned parts) of the seven weights; each[i] unpadded.
size_t layer_weight_bytes(const LayerDims& d, const int* types, size_t* each);
int run_linear(const void* x, int m, int k, int w_type, const void* const* w, const int* n,
               void* const* out, int n_seg, int epi, const void* res, cudaStream_t s);
int layer_forward(kvc_pool* pool, kvc_plan* plan, const int32_t* d_bt, int bt_len, DevBuf& ws,
                  const LayerIO& io, const LayerDims& d, cudaStream_t s);
// The same layer for a decode batch on a paged pool: token i is query i of the
// plan (one new row per sequence, at the plan's position ctx_i - 1); d.seq, d.H,
// d.Hkv and d.D come from the plan and the pool.  Activations live in the plan.
int layer_forward_paged(kvc_pool* pool, kvc_plan* plan, const int32_t* d_bt, int bt_stride,
                        const LayerIO& io, const LayerDims& d, cudaStream_t s);

int pool_alloc(kvc_pool* p, const PoolGeom& g, int device);
void pool_release(kvc_pool* p);
int do_append(kvc_pool* pool, int layer, const void* d_k_new, const void* d_v_new,
              const int32_t* d_bt, int bt_stride, const int32_t* d_rows, const int32_t* d_pos,
              int pos0, int n, cudaStream_t s);
int do_decode(kvc_pool* pool, const kvc_plan* plan, int layer, const void* d_q, void* d_out,
              const int32_t* d_bt, int bt_stride, float scale, cudaStream_t s);
int do_decode_fused(kvc_pool* pool, const kvc_plan* plan, int layer, const void* d_q,
                    void* d_out, const int32_t* d_bt, int bt_stride, float scale,
                    const void* d_k_new, const void* d_v_new, cudaStream_t s,
                    const XchgTarget* xt = nullptr, int early = -1);
// early: -1 = the plan's KVC_PLAN_KV_STABLE flag; 1 = the launch before this one
// (stream order) writes neither KV pages nor block tables, so KV may stream early.
int append_then_decode(kvc_pool* pool, const kvc_plan* plan, int layer, const void* d_q,
                       const void* d_k_new, const void* d_v_new, void* d_out, const int32_t* d_bt,
                       int bt_stride, float scale, cudaStream_t s,
                       const XchgTarget* xt = nullptr, int early = -1);
// Split length (positions) for a batch on a grid of `sms` SMs: see kvc_host.cpp.
int choose_split_tokens(int page_size, const int* ctx, int n_queries, int units_per_split,
                        int sms);
// SM count of `device`; 148 when the query fails (its error is cleared).
int device_sms(int device);
// The split partition of a batch, shared by every planner (kvc_plan_decode and
// kvc_decode_noalloc cut a batch identically): returns the split length C and
// sets refine[i] (n_queries entries) to how many of query i's full splits are cut
// into quarters.  ups = work units per split (KV heads x q-head chunks).
int split_partition(int page_size, const int* ctxs, int n_queries, int ups, int device,
                    int* refine);
// The same for a grid spanning `sms` streaming multiprocessors (no device query).
int split_partition_sms(int page_size, const int* ctxs, int n_queries, int ups, int sms,
                        int* refine);
// The splits of query q (context ctx, split length C, `refine` of its last full
// splits quartered), in position order: emit(int4{q, split, first, end}) for each.
// An empty context has one empty split.  Returns the number of splits.
template <typename Emit>
int emit_splits(int q, int ctx, int C, int refine, Emit&& emit) {
  const int base = ctx > 0 ? (ctx + C - 1) / C : 1;
  const int full = ctx > 0 ? ctx / C : 0;
  int k = 0;
  for (int b = 0; b < base; ++b) {
    const int tb = b * C, te = ctx < (b + 1) * C ? ctx : (b + 1) * C;
    if (b >= full - refine && b < full) {
      for (int j = 0; j < 4; ++j, ++k) emit(make_int4(q, k, tb + j * (C / 4), tb + (j + 1) * (C / 4)));
    } else {
      emit(make_int4(q, k++, tb, te < tb ? tb : te));
    }
  }
  return k;
}
// Plan for q_len queries m = 0..q_len-1 of one sequence (block-table row 0)
// whose context is min(kv_len, start_pos + m + 1) if causal, else kv_len
// (attention.hip:75).
int plan_queries(kvc_plan* plan, const PoolGeom& g, int q_len, int num_heads, int start_pos,
                 int kv_len, bool causal, int device, cudaStream_t s);
}  // namespace kvc
