/*
 * C restatement of gfx1150-inference's decode attention — TEST INFRASTRUCTURE
 * and timed CPU baseline only (tests/, __graft_entry__.smoke(), bench.py's CPU
 * leg).  The product path never links or calls this file.
 *
 * gqa_online_f16 / gqa_online_f32 follow gqa_online_softmax_kernel
 * (src/kernels/attention.hip:35-123) step for step, one (query m, q-head h) at a
 * time:
 *   kv_h = h / (H / Hkv)                                        (:59-60)
 *   max_kv = causal ? min(kv_len, start_pos + m + 1) : kv_len   (:75)
 *   for s < max_kv: dot = q . k_s; score = dot * scale          (:80-99)
 *       m_new = max(m_prev, score); e_prev = exp(m_prev - m_new);
 *       e_cur = exp(score - m_new); l = l * e_prev + e_cur;
 *       acc = acc * e_prev + e_cur * v_s                         (:100-112)
 *   out = acc * (l > 0 ? 1 / l : 0), rounded to fp16             (:115-122)
 * fp16 inputs are widened to fp32; the (m, h) pairs run in parallel with
 * OpenMP, which is where this port differs from the reference's one wave per
 * pair on the GPU.
 *
 * gqa_decode_batch_f16 runs that kernel for a batch of independent sequences
 * (one query each over its own token-major K/V), the way the reference's
 * engine serves a batch one sequence after another (src/inference.py:435-447).
 */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef _Float16 f16;

static void attend_one_f16(const f16* q, const f16* K, const f16* V, f16* out, int kv_len,
                           int max_kv, int Hkv, int D, int kv_h, float scale) {
  float qf[256], acc[256];
  for (int d = 0; d < D; ++d) {
    qf[d] = (float)q[d];
    acc[d] = 0.0f;
  }
  float m_prev = -FLT_MAX, l_prev = 0.0f;
  (void)kv_len;
  for (int s = 0; s < max_kv; ++s) {
    const f16* kp = K + ((size_t)s * Hkv + kv_h) * D;
    const f16* vp = V + ((size_t)s * Hkv + kv_h) * D;
    float dot = 0.0f;
    for (int d = 0; d < D; ++d) dot += qf[d] * (float)kp[d];
    const float score = dot * scale;
    const float m_new = fmaxf(m_prev, score);
    const float e_prev = expf(m_prev - m_new);
    const float e_cur = expf(score - m_new);
    l_prev = l_prev * e_prev + e_cur;
    for (int d = 0; d < D; ++d) acc[d] = acc[d] * e_prev + e_cur * (float)vp[d];
    m_prev = m_new;
  }
  const float inv_l = l_prev > 0.0f ? 1.0f / l_prev : 0.0f;
  for (int d = 0; d < D; ++d) out[d] = (f16)(acc[d] * inv_l);
}

static void attend_one_f32(const float* q, const float* K, const float* V, float* out,
                           int max_kv, int Hkv, int D, int kv_h, float scale) {
  float acc[256];
  for (int d = 0; d < D; ++d) acc[d] = 0.0f;
  float m_prev = -FLT_MAX, l_prev = 0.0f;
  for (int s = 0; s < max_kv; ++s) {
    const float* kp = K + ((size_t)s * Hkv + kv_h) * D;
    const float* vp = V + ((size_t)s * Hkv + kv_h) * D;
    float dot = 0.0f;
    for (int d = 0; d < D; ++d) dot += q[d] * kp[d];
    const float score = dot * scale;
    const float m_new = fmaxf(m_prev, score);
    const float e_prev = expf(m_prev - m_new);
    const float e_cur = expf(score - m_new);
    l_prev = l_prev * e_prev + e_cur;
    for (int d = 0; d < D; ++d) acc[d] = acc[d] * e_prev + e_cur * vp[d];
    m_prev = m_new;
  }
  const float inv_l = l_prev > 0.0f ? 1.0f / l_prev : 0.0f;
  for (int d = 0; d < D; ++d) out[d] = acc[d] * inv_l;
}

/* Returns 0, or -1 for arguments the reference rejects (attention.hip:242-247). */
int gqa_online_f16(const void* Q, const void* K, const void* V, void* Out, int q_len,
                   int kv_len, int H, int Hkv, int D, int start_pos, float scale, int causal,
                   int threads) {
  if (D <= 0 || D > 256 || Hkv <= 0 || H % Hkv != 0) return -1;
  const int group = H / Hkv;
  const long total = (long)q_len * H;
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads > 0 ? threads : 1)
  for (long i = 0; i < total; ++i) {
    const int m = (int)(i / H), h = (int)(i % H);
    int max_kv = causal ? (start_pos + m + 1 < kv_len ? start_pos + m + 1 : kv_len) : kv_len;
    if (max_kv < 0) max_kv = 0;
    attend_one_f16((const f16*)Q + ((size_t)m * H + h) * D, (const f16*)K, (const f16*)V,
                   (f16*)Out + ((size_t)m * H + h) * D, kv_len, max_kv, Hkv, D, h / group, scale);
  }
  return 0;
}

int gqa_online_f32(const float* Q, const float* K, const float* V, float* Out, int q_len,
                   int kv_len, int H, int Hkv, int D, int start_pos, float scale, int causal,
                   int threads) {
  if (D <= 0 || D > 256 || Hkv <= 0 || H % Hkv != 0) return -1;
  const int group = H / Hkv;
  const long total = (long)q_len * H;
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads > 0 ? threads : 1)
  for (long i = 0; i < total; ++i) {
    const int m = (int)(i / H), h = (int)(i % H);
    int max_kv = causal ? (start_pos + m + 1 < kv_len ? start_pos + m + 1 : kv_len) : kv_len;
    if (max_kv < 0) max_kv = 0;
    attend_one_f32(Q + ((size_t)m * H + h) * D, K, V, Out + ((size_t)m * H + h) * D, max_kv, Hkv,
                   D, h / group, scale);
  }
  return 0;
}

/* Batch of n sequences, one query each: Q (n, H, D); K[i], V[i] point at
 * sequence i's token-major rows (ctx[i], Hkv, D); Out (n, H, D). */
int gqa_decode_batch_f16(int n, const void* Q, const void* const* K, const void* const* V,
                         const int* ctx, void* Out, int H, int Hkv, int D, float scale,
                         int threads) {
  if (D <= 0 || D > 256 || Hkv <= 0 || H % Hkv != 0) return -1;
  const int group = H / Hkv;
  const long total = (long)n * H;
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads > 0 ? threads : 1)
  for (long i = 0; i < total; ++i) {
    const int sq = (int)(i / H), h = (int)(i % H);
    attend_one_f16((const f16*)Q + ((size_t)sq * H + h) * D, (const f16*)K[sq],
                   (const f16*)V[sq], (f16*)Out + ((size_t)sq * H + h) * D, ctx[sq], ctx[sq],
                   Hkv, D, h / group, scale);
  }
  return 0;
}

int gqa_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
