/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for packed variable-length attention.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load this
 * library, and only as the checker or the timed CPU baseline. The product path
 * (packed_encoders_b200) never calls it; there is no CPU fallback.
 *
 * What it restates (fp32 inputs, fp32 outputs, double-precision reductions):
 *
 *   for every sequence s = [cu[s], cu[s+1]) and every query head h,
 *   query token i of s reads the keys j of s allowed by the band
 *       (i - j) <= window_left   when window_left  >= 0        (left context)
 *       (j - i) <= window_right  when window_right >= 0        (right context)
 *       j <= i                   when causal                  (right context 0)
 *   out[i,h,:] = sum_j softmax_j(scale * q[i,h,:] . k[j,h/G,:]) * v[j,h/G,:]
 *   lse[h,i]   = log(sum_j exp(scale * q[i,h,:] . k[j,h/G,:]))   (natural log)
 *   with G = heads / kv_heads query heads per key/value head (GQA).
 *
 * Reference behaviour it follows (packed-encoders 0.3.0):
 *   - per-row key window [max(0, p-half), min(len, p+half+1)):
 *       packed_encoders/cpu/local_attention_x86.c:132-157 (tile_attention) and
 *       :144-149 (first/last per row); global attention is half >= longest (:206)
 *   - softmax as exp(s - rowmax) / sum: local_attention_x86.c:72-91 (softmax_row)
 *   - scores scaled after the dot product: local_attention_x86.c:55 (0.125 = 64**-0.5)
 *   - the band for causal / (left, right) windows, queries aligned to the END of the key
 *     segment for the prefixed form: packed_encoders/runtime/attention.py:157-170 (_band)
 *   - per-segment evaluation with GQA by repeat_interleave of K/V heads, empty segments
 *     skipped: runtime/attention.py:99-101 (_repeat_kv), :173-184 (_segments)
 *   - Triton kernel masks (|i-j| <= half, keys inside the sequence):
 *       packed_encoders/_kernels/triton_packed_attention.py:98-143
 *   - argument validation returning negative status codes, no exit/trap:
 *       local_attention_x86.c:196-211
 *
 * Layout: token-major q [Tq, H, D], k/v [Tk, KV, D], out [Tq, H, D], all fp32 with the
 * given element strides (token, head); D is contiguous. lse (optional) is [H, Tq].
 * Queries of segment s are rows cu_q[s]..cu_q[s+1]; its keys cu_k[s]..cu_k[s+1]. When the
 * query segment is shorter than the key segment (the reference's prefixed form) the
 * queries are the LAST rows of the key segment: query r sits at key position
 * r + (len_k - len_q).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define ORACLE_OK 0
#define ORACLE_EINVAL (-1)
#define ORACLE_ENOMEM (-2)

int oracle_version(void) { return 1; }

/* One (segment, head) task: len_q query rows against len_k key rows. */
static void segment_head(const float *q, const float *k, const float *v, float *out, float *lse,
                         long q_tok, long q_head, long k_tok, long k_head, long v_tok, long v_head,
                         long o_tok, long o_head, int dim, int len_q, int len_k, int q0, int k0,
                         int head, int kv_head, long lse_row, float scale, int window_left,
                         int window_right, int causal, double *scores, double *acc) {
    int shift = len_k - len_q; /* query r is key position r + shift */
    int right = causal ? 0 : window_right;
    for (int r = 0; r < len_q; ++r) {
        int p = r + shift;
        int lo = 0, hi = len_k; /* allowed keys [lo, hi) */
        if (window_left >= 0 && p - window_left > lo) lo = p - window_left;
        if (right >= 0 && p + right + 1 < hi) hi = p + right + 1;
        const float *qr = q + (long)(q0 + r) * q_tok + (long)head * q_head;
        float *orow = out + (long)(q0 + r) * o_tok + (long)head * o_head;
        if (hi <= lo) { /* no key allowed: zero output, -inf lse (never happens for p in range) */
            for (int d = 0; d < dim; ++d) orow[d] = 0.f;
            if (lse) lse[lse_row + q0 + r] = -INFINITY;
            continue;
        }
        double m = -INFINITY;
        for (int j = lo; j < hi; ++j) {
            const float *kr = k + (long)(k0 + j) * k_tok + (long)kv_head * k_head;
            double s = 0.0;
            for (int d = 0; d < dim; ++d) s += (double)qr[d] * (double)kr[d];
            s *= (double)scale;
            scores[j - lo] = s;
            if (s > m) m = s;
        }
        double l = 0.0;
        for (int d = 0; d < dim; ++d) acc[d] = 0.0;
        for (int j = lo; j < hi; ++j) {
            double e = exp(scores[j - lo] - m);
            l += e;
            const float *vr = v + (long)(k0 + j) * v_tok + (long)kv_head * v_head;
            for (int d = 0; d < dim; ++d) acc[d] += e * (double)vr[d];
        }
        for (int d = 0; d < dim; ++d) orow[d] = (float)(acc[d] / l);
        if (lse) lse[lse_row + q0 + r] = (float)(m + log(l));
    }
}

/*
 * Packed attention with separate query / key segment boundaries (cu_q, cu_k: int32
 * [n_seq + 1], non-decreasing, cu_q[n_seq] = tokens_q, cu_k[n_seq] = tokens_k, every
 * query segment no longer than its key segment). Returns 0, or a negative code on an
 * invalid argument (nothing written).
 */
int oracle_attention_prefixed(const float *q, const float *k, const float *v, float *out, float *lse,
                              const int32_t *cu_q, const int32_t *cu_k, int n_seq, int tokens_q,
                              int tokens_k, int heads, int kv_heads, int dim, long q_tok, long q_head,
                              long k_tok, long k_head, long v_tok, long v_head, long o_tok, long o_head,
                              float scale, int window_left, int window_right, int causal, int threads) {
    if (!cu_q || !cu_k) return ORACLE_EINVAL;
    if ((tokens_q > 0 && (!q || !out)) || (tokens_k > 0 && (!k || !v))) return ORACLE_EINVAL;
    if (n_seq < 0 || tokens_q < 0 || tokens_k < 0 || heads < 1 || kv_heads < 1 || dim < 1)
        return ORACLE_EINVAL;
    if (heads % kv_heads) return ORACLE_EINVAL;
    if (cu_q[0] != 0 || cu_k[0] != 0 || cu_q[n_seq] != tokens_q || cu_k[n_seq] != tokens_k)
        return ORACLE_EINVAL;
    int longest = 0;
    for (int s = 0; s < n_seq; ++s) {
        int lq = cu_q[s + 1] - cu_q[s], lk = cu_k[s + 1] - cu_k[s];
        if (lq < 0 || lk < 0 || lq > lk) return ORACLE_EINVAL;
        if (lk > longest) longest = lk;
    }
    int group = heads / kv_heads;
    long tasks = (long)n_seq * heads;
    if (threads < 1) threads = 1;
    int failed = 0;
#pragma omp parallel num_threads(threads) if (threads > 1)
    {
        double *scores = (double *)malloc(sizeof(double) * (size_t)(longest > 0 ? longest : 1));
        double *acc = (double *)malloc(sizeof(double) * (size_t)dim);
        if (!scores || !acc) {
#pragma omp atomic write
            failed = 1;
        }
#pragma omp for schedule(dynamic, 1)
        for (long task = 0; task < tasks; ++task) {
            if (!scores || !acc) continue;
            int s = (int)(task / heads), h = (int)(task % heads);
            segment_head(q, k, v, out, lse, q_tok, q_head, k_tok, k_head, v_tok, v_head, o_tok, o_head, dim,
                         cu_q[s + 1] - cu_q[s], cu_k[s + 1] - cu_k[s], cu_q[s], cu_k[s], h, h / group,
                         (long)h * tokens_q, scale, window_left, window_right, causal, scores, acc);
        }
        free(scores);
        free(acc);
    }
    return failed ? ORACLE_ENOMEM : ORACLE_OK;
}

/* Self attention over one set of boundaries (the packed form). */
int oracle_attention(const float *q, const float *k, const float *v, float *out, float *lse,
                     const int32_t *cu_seqlens, int n_seq, int tokens, int heads, int kv_heads, int dim,
                     long q_tok, long q_head, long k_tok, long k_head, long v_tok, long v_head, long o_tok,
                     long o_head, float scale, int window_left, int window_right, int causal, int threads) {
    return oracle_attention_prefixed(q, k, v, out, lse, cu_seqlens, cu_seqlens, n_seq, tokens, tokens, heads,
                                     kv_heads, dim, q_tok, q_head, k_tok, k_head, v_tok, v_head, o_tok, o_head,
                                     scale, window_left, window_right, causal, threads);
}

/*
 * Useful (allowed) query-key pairs of one head, summed over the segments: the numerator
 * of the useful-pair FLOP count 4 * pairs * heads * dim. Same band as above.
 */
long long oracle_useful_pairs(const int32_t *cu_seqlens, int n_seq, int window_left, int window_right,
                              int causal) {
    long long pairs = 0;
    int right = causal ? 0 : window_right;
    for (int s = 0; s < n_seq; ++s) {
        int len = cu_seqlens[s + 1] - cu_seqlens[s];
        for (int p = 0; p < len; ++p) {
            int lo = 0, hi = len;
            if (window_left >= 0 && p - window_left > lo) lo = p - window_left;
            if (right >= 0 && p + right + 1 < hi) hi = p + right + 1;
            if (hi > lo) pairs += hi - lo;
        }
    }
    return pairs;
}
