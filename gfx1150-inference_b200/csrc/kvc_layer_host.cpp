// Host side of the layer pipeline: the projections, RMSNorm and the whole layer of
// forward_layer_cached (bindings.cpp:562-627 ⇒ launch_forward_layer_cached_fp16,
// attention.hip:603-695) over the device KV pool.
//
// One layer on the device: RMSNorm → q/k/v projections (one launch when the three
// weights share a type) → RoPE on q and the new K rows → append + attention (the
// fused decode kernel for one token; append then attend for a prefill chunk) →
// output projection → residual + RMSNorm → gate/up projections with the SwiGLU in
// their epilogue → down projection with the residual in its epilogue.
//
// The same layer runs for a batch of sequences on a paged pool
// (kvc_forward_layer_paged, the batched form of generate_batch_ids'
// one-sequence-at-a-time loop, inference.py:435-447): one token per query of a
// decode plan, rotated at the plan's positions, appended into its block-table row.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "kvc_common.h"
#include "kvc_internal.h"
#include "kvcache.h"

namespace kvc {

namespace {
size_t al256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }
}  // namespace

int check_weight(int w_type, int n, int k, const char* name) {
  int per = 0, bytes = 0;
  weight_block(w_type, &per, &bytes);
  if (per == 0)
    return set_error(KVC_ERR_INVALID_ARG, "Unsupported weight type %d for %s.", w_type, name);
  if (k <= 0 || k % per != 0)
    return set_error(KVC_ERR_INVALID_ARG, "%s K must be divisible by %d for weight type %d.",
                     name, per, w_type);
  // limits of the tensor-core projection kernel (all Llama-family shapes meet them)
  if (k % 32 != 0)
    return set_error(KVC_ERR_INVALID_ARG, "%s K must be a multiple of 32.", name);
  if (n <= 0 || n % 16 != 0)
    return set_error(KVC_ERR_INVALID_ARG, "%s output features must be a positive multiple of 16.",
                     name);
  return KVC_OK;
}

size_t weight_size(int w_type, int n, int k) {
  int per = 0, bytes = 0;
  weight_block(w_type, &per, &bytes);
  return per ? static_cast<size_t>(n) * (k / per) * bytes : 0;
}

int run_linear(const void* x, int m, int k, int w_type, const void* const* w, const int* n,
               void* const* out, int n_seg, int epi, const void* res, cudaStream_t s) {
  if (m < 0) return set_error(KVC_ERR_INVALID_ARG, "m must be non-negative.");
  if (m == 0) return KVC_OK;
  if (!x || (epi == kEpiResidual && !res))
    return set_error(KVC_ERR_INVALID_ARG, "activations must not be null.");
  if (reinterpret_cast<uintptr_t>(x) & 15u)
    return set_error(KVC_ERR_INVALID_ARG, "activations must be 16-byte aligned.");
  LinearArgs a;
  a.x = static_cast<const __half*>(x);
  a.x_ld = k;
  a.m = m;
  a.k = k;
  a.w_type = w_type;
  a.row_bytes = weight_size(w_type, 1, k);
  a.n_seg = n_seg;
  a.epi = epi;
  a.res = static_cast<const __half*>(res);
  for (int i = 0; i < n_seg; ++i) {
    if (int rc = check_weight(w_type, n[i], k, "weight")) return rc;
    if (!w[i] || !out[i]) return set_error(KVC_ERR_INVALID_ARG, "weights and outputs must not be null.");
    if (reinterpret_cast<uintptr_t>(w[i]) & 15u)
      return set_error(KVC_ERR_INVALID_ARG, "weights must be 16-byte aligned.");
    if (reinterpret_cast<uintptr_t>(out[i]) & 1u)
      return set_error(KVC_ERR_INVALID_ARG, "outputs must be 2-byte aligned.");
    a.seg[i].w = static_cast<const uint8_t*>(w[i]);
    a.seg[i].out = static_cast<__half*>(out[i]);
    a.seg[i].n = n[i];
    a.seg[i].out_ld = n[i];
  }
  if (epi == kEpiSwiglu && (n_seg != 2 || n[0] != n[1]))
    return set_error(KVC_ERR_INVALID_ARG, "gate and up must have the same shape.");
  cudaError_t e = launch_linear(a, s);
  if (e != cudaSuccess) return cuda_error(e, "linear kernel");
  return KVC_OK;
}

int check_layer(const LayerDims& d, const int* types) {
  if (d.seq < 0 || d.pos < 0) return set_error(KVC_ERR_INVALID_ARG, "seq_len and pos_offset must be non-negative.");
  if (d.hidden <= 0 || d.inter <= 0 || d.H <= 0 || d.Hkv <= 0 || d.D <= 0)
    return set_error(KVC_ERR_INVALID_ARG, "layer dimensions must be positive.");
  if (d.H % d.Hkv != 0)
    return set_error(KVC_ERR_INVALID_ARG, "num_heads must be divisible by num_kv_heads.");
  if (d.D % 2 != 0 || d.D > 2 * kMaxRopePairs)
    return set_error(KVC_ERR_INVALID_ARG, "head_dim must be even and at most %d.", 2 * kMaxRopePairs);
  const int qd = d.H * d.D, kd = d.Hkv * d.D;
  // bindings.cpp:601-607: (name, N, K) of each weight
  const char* names[7] = {"wq", "wk", "wv", "wo", "wgate", "wup", "wdown"};
  const int ns[7] = {qd, kd, kd, d.hidden, d.inter, d.inter, d.hidden};
  const int ks[7] = {d.hidden, d.hidden, d.hidden, qd, d.hidden, d.hidden, d.inter};
  for (int i = 0; i < 7; ++i)
    if (int rc = check_weight(types[i], ns[i], ks[i], names[i])) return rc;
  if (d.hidden % 8 != 0) return set_error(KVC_ERR_INVALID_ARG, "hidden_size must be a multiple of 8.");
  return KVC_OK;
}

size_t layer_weight_bytes(const LayerDims& d, const int* types, size_t* each) {
  const int qd = d.H * d.D, kd = d.Hkv * d.D;
  const int ns[7] = {qd, kd, kd, d.hidden, d.inter, d.inter, d.hidden};
  const int ks[7] = {d.hidden, d.hidden, d.hidden, qd, d.hidden, d.hidden, d.inter};
  size_t tot = 0;
  for (int i = 0; i < 7; ++i) {
    each[i] = weight_size(types[i], ns[i], ks[i]);
    tot += al256(each[i]);
  }
  return tot;
}

namespace {

// The layer around its attention step: RMSNorm, the q/k/v projections, then
// attend(q, k, v, qr, kr, attn) — which rotates q and the new K rows into qr / kr,
// appends them with the V rows and attends into attn — then the output
// projection, residual + RMSNorm, gate/up with the SwiGLU and the down
// projection with the second residual.  d.seq rows of io.x_in, one per token.
template <class Attend>
int layer_steps(DevBuf& ws, const LayerIO& io, const LayerDims& d, cudaStream_t s,
                Attend&& attend) {
  const int seq = d.seq, qd = d.H * d.D, kd = d.Hkv * d.D;
  if (seq == 0) return KVC_OK;
  const size_t hb = sizeof(__half) * seq * d.hidden, qb = sizeof(__half) * seq * qd;
  const size_t kb = sizeof(__half) * seq * kd, ib = sizeof(__half) * seq * d.inter;
  const size_t need = 4 * al256(hb) + 3 * al256(qb) + 3 * al256(kb) + 2 * al256(ib);
  cudaError_t e = ws.ensure(need);
  if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(layer workspace)");
  uint8_t* p = static_cast<uint8_t*>(ws.ptr);
  auto take = [&](size_t b) {
    __half* r = reinterpret_cast<__half*>(p);
    p += al256(b);
    return r;
  };
  __half *normed = take(hb), *q = take(qb), *k = take(kb), *v = take(kb), *qr = take(qb);
  __half *kr = take(kb), *attn = take(qb), *proj = take(hb), *h = take(hb), *nh = take(hb);
  __half *act = take(ib), *up = take(ib);
  int rc;
  // 1. pre-attention RMSNorm (attention.hip:643)
  if ((e = launch_rmsnorm(io.x_in, nullptr, io.attn_norm, nullptr, normed, seq, d.hidden, d.eps, s)))
    return cuda_error(e, "rmsnorm kernel");
  // 2. q, k, v projections (attention.hip:650-652); equal types share one launch
  {
    const void* w[3] = {io.w[0], io.w[1], io.w[2]};
    const int n[3] = {qd, kd, kd};
    void* out[3] = {q, k, v};
    int i = 0;
    while (i < 3) {
      int j = i + 1;
      while (j < 3 && io.type[j] == io.type[i]) ++j;
      if ((rc = run_linear(normed, seq, d.hidden, io.type[i], w + i, n + i, out + i, j - i,
                           kEpiStore, nullptr, s)))
        return rc;
      i = j;
    }
  }
  // 3-5. RoPE, append, attention (attention.hip:655-668)
  if ((rc = attend(q, k, v, qr, kr, attn))) return rc;
  // 6. output projection (attention.hip:671)
  {
    const void* w[1] = {io.w[3]};
    const int n[1] = {d.hidden};
    void* out[1] = {proj};
    if ((rc = run_linear(attn, seq, qd, io.type[3], w, n, out, 1, kEpiStore, nullptr, s))) return rc;
  }
  // 7. residual + RMSNorm (attention.hip:679-681)
  if ((e = launch_rmsnorm(io.x_in, proj, io.ffn_norm, h, nh, seq, d.hidden, d.eps, s)))
    return cuda_error(e, "rmsnorm kernel");
  // 8. gate and up with the SwiGLU (attention.hip:684-686)
  if (io.type[4] == io.type[5]) {
    const void* w[2] = {io.w[4], io.w[5]};
    const int n[2] = {d.inter, d.inter};
    void* out[2] = {act, act};
    if ((rc = run_linear(nh, seq, d.hidden, io.type[4], w, n, out, 2, kEpiSwiglu, nullptr, s)))
      return rc;
  } else {
    for (int i = 0; i < 2; ++i) {
      const void* w[1] = {io.w[4 + i]};
      const int n[1] = {d.inter};
      void* out[1] = {i == 0 ? act : up};
      if ((rc = run_linear(nh, seq, d.hidden, io.type[4 + i], w, n, out, 1, kEpiStore, nullptr, s)))
        return rc;
    }
    if ((e = launch_swiglu(act, up, act, static_cast<size_t>(seq) * d.inter, s)))
      return cuda_error(e, "swiglu kernel");
  }
  // 9. down projection with the second residual (attention.hip:687-689)
  {
    const void* w[1] = {io.w[6]};
    const int n[1] = {d.hidden};
    void* out[1] = {io.x_out};
    if ((rc = run_linear(act, seq, d.inter, io.type[6], w, n, out, 1, kEpiResidual, h, s))) return rc;
  }
  return KVC_OK;
}

// RoPE arguments for q (d.H heads) and the new K rows (d.Hkv heads) of d.seq tokens.
RopeArgs rope_args(const LayerDims& d, const __half* q, const __half* k, __half* qr, __half* kr) {
  RopeArgs ra{};
  ra.src[0] = reinterpret_cast<const uint8_t*>(q);
  ra.dst[0] = reinterpret_cast<uint8_t*>(qr);
  ra.heads[0] = d.H;
  ra.src[1] = reinterpret_cast<const uint8_t*>(k);
  ra.dst[1] = reinterpret_cast<uint8_t*>(kr);
  ra.heads[1] = d.Hkv;
  ra.n_tokens = d.seq;
  ra.head_dim = d.D;
  ra.dtype = KVC_DTYPE_F16;
  ra.neox = d.neox ? 1 : 0;
  rope_inv_freq(d.base, d.D, ra.inv_freq);
  return ra;
}

}  // namespace

int layer_forward(kvc_pool* pool, kvc_plan* plan, const int32_t* d_bt, int bt_len, DevBuf& ws,
                  const LayerIO& io, const LayerDims& d, cudaStream_t s) {
  if (pool->g.dtype != KVC_DTYPE_F16)
    return set_error(KVC_ERR_INVALID_ARG, "forward_layer_cached needs an fp16 KV pool.");
  return layer_steps(ws, io, d, s, [&](const __half* q, const __half* k, const __half* v,
                                       __half* qr, __half* kr, __half* attn) -> int {
    // the attention plan first: its upload must not sit between RoPE and the decode
    int rc = cached_plan(pool, plan, d.seq, d.pos, d.H, true, s);
    if (rc) return rc;
    // RoPE on q and the new K rows at pos_offset.. (attention.hip:655-660)
    RopeArgs ra = rope_args(d, q, k, qr, kr);
    ra.pos0 = d.pos;
    ra.positions = nullptr;
    const bool one = d.seq == 1;
    cudaError_t e = launch_rope(ra, s, one);
    if (e) return cuda_error(e, "rope kernel");
    // append the rotated K rows and V rows, attend (attention.hip:663-668)
    return cached_run(pool, plan, d_bt, bt_len, qr, kr, v, attn, d.layer, d.seq, d.pos, d.scale,
                      s, one ? 1 : -1);
  });
}

int layer_forward_paged(kvc_pool* pool, kvc_plan* plan, const int32_t* d_bt, int bt_stride,
                        const LayerIO& io, const LayerDims& d, cudaStream_t s) {
  return layer_steps(plan->d_layer, io, d, s, [&](const __half* q, const __half* k,
                                                  const __half* v, __half* qr, __half* kr,
                                                  __half* attn) -> int {
    // RoPE at each query's own position (the plan's ctx - 1), as a programmatic
    // dependent that lets the decode behind it start streaming KV; it writes only
    // qr / kr.  Then the fused append + attention of every sequence.
    RopeArgs ra = rope_args(d, q, k, qr, kr);
    ra.positions = plan->dev_pos;
    cudaError_t e = launch_rope(ra, s, true);
    if (e) return cuda_error(e, "rope kernel");
    return append_then_decode(pool, plan, d.layer, qr, kr, v, attn, d_bt, bt_stride, d.scale, s,
                              nullptr, 1);
  });
}

}  // namespace kvc

using namespace kvc;

extern "C" int kvc_weight_bytes(int w_type, int n, int k, size_t* out) {
  if (!out) return set_error(KVC_ERR_INVALID_ARG, "out must not be null.");
  int per = 0, bytes = 0;
  weight_block(w_type, &per, &bytes);
  if (per == 0) return set_error(KVC_ERR_INVALID_ARG, "Unsupported weight type %d.", w_type);
  if (n < 0 || k <= 0 || k % per != 0)
    return set_error(KVC_ERR_INVALID_ARG, "K must be divisible by %d for weight type %d.", per, w_type);
  *out = weight_size(w_type, n, k);
  return KVC_OK;
}

extern "C" int kvc_linear(const void* d_x, int m, int k, const void* d_w, int w_type, int n,
                          void* d_out, void* stream) {
  const void* w[1] = {d_w};
  const int ns[1] = {n};
  void* out[1] = {d_out};
  return run_linear(d_x, m, k, w_type, w, ns, out, 1, kEpiStore, nullptr,
                    static_cast<cudaStream_t>(stream));
}

extern "C" int kvc_linear_swiglu(const void* d_x, int m, int k, const void* d_w_gate,
                                 const void* d_w_up, int w_type, int n, void* d_out,
                                 void* stream) {
  const void* w[2] = {d_w_gate, d_w_up};
  const int ns[2] = {n, n};
  void* out[2] = {d_out, d_out};
  return run_linear(d_x, m, k, w_type, w, ns, out, 2, kEpiSwiglu, nullptr,
                    static_cast<cudaStream_t>(stream));
}

extern "C" int kvc_linear_residual(const void* d_x, int m, int k, const void* d_w, int w_type,
                                   int n, const void* d_res, void* d_out, void* stream) {
  const void* w[1] = {d_w};
  const int ns[1] = {n};
  void* out[1] = {d_out};
  return run_linear(d_x, m, k, w_type, w, ns, out, 1, kEpiResidual, d_res,
                    static_cast<cudaStream_t>(stream));
}

extern "C" int kvc_rmsnorm(const void* d_x, const void* d_res, void* d_h_out, const void* d_w,
                           void* d_out, int m, int k, float eps, void* stream) {
  if (m < 0 || k <= 0) return set_error(KVC_ERR_INVALID_ARG, "m must be non-negative and k positive.");
  if (!d_x || !d_w || !d_out || (d_res && !d_h_out))
    return set_error(KVC_ERR_INVALID_ARG, "buffers must not be null.");
  cudaError_t e = launch_rmsnorm(static_cast<const __half*>(d_x), static_cast<const __half*>(d_res),
                                 static_cast<const __half*>(d_w), static_cast<__half*>(d_h_out),
                                 static_cast<__half*>(d_out), m, k, eps,
                                 static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? KVC_OK : cuda_error(e, "rmsnorm kernel");
}

extern "C" int kvc_forward_layer_paged(
    kvc_pool_t* pool, const kvc_plan_t* plan, int layer_idx, const void* d_x_in, void* d_x_out,
    const void* d_attn_norm_w, const void* d_wq, int wq_type, const void* d_wk, int wk_type,
    const void* d_wv, int wv_type, const void* d_wo, int wo_type, const void* d_ffn_norm_w,
    const void* d_wgate, int wgate_type, const void* d_wup, int wup_type, const void* d_wdown,
    int wdown_type, const int32_t* d_block_tables, int bt_stride, int hidden_size,
    int intermediate_size, float rms_norm_eps, float rope_freq_base, int rope_neox, float scale,
    void* stream) {
  if (!pool || !plan) return set_error(KVC_ERR_INVALID_ARG, "pool and plan must not be null.");
  if (!plan->valid) return set_error(KVC_ERR_INVALID_ARG, "plan has not been built.");
  const PoolGeom& g = pool->g;
  if (g.dtype != KVC_DTYPE_F16)
    return set_error(KVC_ERR_INVALID_ARG, "the layer pipeline needs an fp16 KV pool.");
  if (layer_idx < 0 || layer_idx >= g.num_layers)
    return set_error(KVC_ERR_OUT_OF_RANGE, "layer_idx out of range for the KV pool.");
  if (plan->head_dim != g.head_dim || plan->num_kv_heads != g.num_kv_heads ||
      plan->page_size != g.page_size)
    return set_error(KVC_ERR_INVALID_ARG, "plan was built for a pool of another geometry.");
  LayerDims d;
  d.layer = layer_idx;
  d.seq = plan->n_queries;
  d.pos = 0;
  d.hidden = hidden_size;
  d.inter = intermediate_size;
  d.H = plan->num_heads;
  d.Hkv = g.num_kv_heads;
  d.D = g.head_dim;
  d.eps = rms_norm_eps;
  d.base = rope_freq_base;
  d.scale = scale;
  d.neox = rope_neox != 0;
  const int types[7] = {wq_type, wk_type, wv_type, wo_type, wgate_type, wup_type, wdown_type};
  const void* w[7] = {d_wq, d_wk, d_wv, d_wo, d_wgate, d_wup, d_wdown};
  int rc = check_layer(d, types);
  if (rc) return rc;
  if (!(rope_freq_base > 0.0f))
    return set_error(KVC_ERR_INVALID_ARG, "rope_freq_base must be positive.");
  for (int32_t c : plan->positions)
    if (c < 0) return set_error(KVC_ERR_INVALID_ARG, "a query with an empty context has no new row.");
  if (d.seq == 0) return KVC_OK;
  if (!d_x_in || !d_x_out || !d_attn_norm_w || !d_ffn_norm_w || !d_block_tables)
    return set_error(KVC_ERR_INVALID_ARG, "device buffers must not be null.");
  LayerIO io;
  for (int i = 0; i < 7; ++i) {
    if (!w[i]) return set_error(KVC_ERR_INVALID_ARG, "weight buffers must not be null.");
    io.w[i] = w[i];
    io.type[i] = types[i];
  }
  io.x_in = static_cast<const __half*>(d_x_in);
  io.x_out = static_cast<__half*>(d_x_out);
  io.attn_norm = static_cast<const __half*>(d_attn_norm_w);
  io.ffn_norm = static_cast<const __half*>(d_ffn_norm_w);
  if (const int rc_dev = use_device(pool->device)) return rc_dev;
  return layer_forward_paged(pool, const_cast<kvc_plan*>(plan), d_block_tables, bt_stride, io, d,
                             static_cast<cudaStream_t>(stream));
}
