/*
 * pmkl_oracle.c -- CPU restatement of the reference's arithmetic for the
 * causal-attention and warp-softmax path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (the CUDA library, the
 * torch binding, the C++ shim) links, loads or calls this file.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg use it, and only as
 * the checker / the timed CPU baseline.
 *
 * Every function restates one reference function in plain C, keeping the
 * reference's operation order and accumulation types so that, compiled with
 * the same flags as the reference, results match it bit for bit in fp32:
 *
 *   pmkl_oracle_attention_fwd_f32
 *       pmkl_pytorch_ext/fused_self_attention.cpp:5-64
 *       (pmkl_cpu::host_self_attention_forward<float>; the identical
 *        test/test_causal_attention.cpp:11-70 is the GPU test's oracle)
 *   pmkl_oracle_attention_rows_f32
 *       the same recurrence evaluated only on a caller-chosen list of query
 *       rows.  A causal row i depends only on K/V rows [0, i], so a sampled row
 *       equals the full computation's row.  Used at the large benchmark
 *       shapes, where the reference's S x S scratch and O(S^2 D) single-thread
 *       loop would take hours.
 *   pmkl_oracle_attention_bwd_exact_f32
 *       pmkl_pytorch_ext/fused_self_attention.cpp:66-135
 *       (pmkl_cpu::host_self_attention_backward<float>), O(S^3 D) as written
 *   pmkl_oracle_attention_bwd_f32
 *       the same gradient reduced to O(S^2 D) (double accumulation), for the
 *       larger parity cases; checked against the exact form in tests
 *   pmkl_oracle_softmax_fwd_f32
 *       test/test_softmax.cpp:10-28 (host_softmax_forward<float,float,float>)
 *   pmkl_oracle_log_softmax_fwd_f32
 *       pmkl/norm/warp_softmax.h:120-150 with is_log_softmax = true: the
 *       reference ships no host log-softmax, so this restates the device
 *       kernel's formula  x - max - log(sum(exp(x - max))).
 *
 * Differences from the reference that do not change results:
 *   - the reference allocates an S x S float scratch per (batch, head)
 *     (fused_self_attention.cpp:22); here one row of S floats is enough,
 *     because each output row only reads its own score row;
 *   - the reference hard-codes scale = 1.0f / sqrt((float)D)
 *     (fused_self_attention.cpp:30); here the caller passes the scale, and
 *     passing exactly that value reproduces the reference.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* One query row of fused_self_attention.cpp:23-61.  `srow` is scratch of
 * length S.  Returns nothing; writes o_row[D], *m_out, *l_out. */
static void attention_row(const float *q_b, const float *k_b, const float *v_b,
                          int S, int D, int causal, float scale, int row,
                          float *srow, float *o_row, float *m_out,
                          float *l_out) {
    const float neg_inf = -INFINITY;
    const float *q_s = q_b + (int64_t)row * D;
    /* scores: float accumulation in kk order, then times scale (:23-32) */
    for (int n = 0; n < S; n++) {
        const float *k_s = k_b + (int64_t)n * D;
        float sum = 0.0f;
        for (int kk = 0; kk < D; kk++) sum += q_s[kk] * k_s[kk];
        srow[n] = sum * scale;
    }
    /* causal mask to -inf (:33-37) */
    if (causal)
        for (int n = row + 1; n < S; n++) srow[n] = neg_inf;
    /* max in float, exp-sum in double (:38-52) */
    float max_value = neg_inf;
    for (int n = 0; n < S; n++) max_value = srow[n] > max_value ? srow[n] : max_value;
    *m_out = max_value;
    double e2sum = 0.0;
    for (int n = 0; n < S; n++) e2sum += exp((double)srow[n] - max_value);
    *l_out = (float)e2sum;
    /* p = exp(float) / double, stored back to float (:49-51) */
    for (int n = 0; n < S; n++) srow[n] = (float)(expf(srow[n] - max_value) / e2sum);
    /* P V with float accumulation in key order (:53-61) */
    for (int kk = 0; kk < D; kk++) {
        float sum = 0.0f;
        for (int n = 0; n < S; n++) sum += srow[n] * v_b[(int64_t)n * D + kk];
        o_row[kk] = sum;
    }
}

/* q, k, v, o: [BH, S, D] contiguous fp32.  m, l: [BH, S].  Returns 0, or -1
 * when the scratch row cannot be allocated. */
int pmkl_oracle_attention_fwd_f32(const float *q, const float *k, const float *v,
                                  float *o, float *m, float *l, int64_t BH, int S,
                                  int D, int causal, float scale) {
    if (BH <= 0 || S <= 0 || D <= 0) return 0;
    float *srow = (float *)malloc(sizeof(float) * (size_t)S);
    if (!srow) return -1;
    for (int64_t b = 0; b < BH; b++) {
        const int64_t off = b * (int64_t)S * D;
        for (int row = 0; row < S; row++)
            attention_row(q + off, k + off, v + off, S, D, causal, scale, row, srow,
                          o + off + (int64_t)row * D, m + b * S + row, l + b * S + row);
    }
    free(srow);
    return 0;
}

/* Sampled rows: for each i in [0, nrows), evaluates query row rows[i] of
 * slice slices[i].  Outputs are packed: o[nrows, D], m[nrows], l[nrows]. */
int pmkl_oracle_attention_rows_f32(const float *q, const float *k, const float *v,
                                   int S, int D, int causal, float scale,
                                   const int64_t *slices, const int32_t *rows,
                                   int64_t nrows, float *o, float *m, float *l) {
    float *srow = (float *)malloc(sizeof(float) * (size_t)(S > 0 ? S : 1));
    if (!srow) return -1;
    for (int64_t i = 0; i < nrows; i++) {
        const int64_t off = slices[i] * (int64_t)S * D;
        attention_row(q + off, k + off, v + off, S, D, causal, scale, rows[i], srow,
                      o + i * D, m + i, l + i);
    }
    free(srow);
    return 0;
}

/* test/test_softmax.cpp:10-28 with output_t = input_t = acc_t = float. */
void pmkl_oracle_softmax_fwd_f32(float *dst, const float *src, int elements,
                                 int stride, int rows) {
    for (int b = 0; b < rows; b++) {
        const float *src_b = src + (int64_t)b * stride;
        float *dst_b = dst + (int64_t)b * stride;
        float max_v = -99999999;
        for (int i = 0; i < elements; i++) max_v = src_b[i] > max_v ? src_b[i] : max_v;
        float sum = 0;
        for (int i = 0; i < elements; i++) sum += expf(src_b[i] - max_v);
        for (int i = 0; i < elements; i++) dst_b[i] = expf(src_b[i] - max_v) / sum;
    }
}

/* Log-softmax as pmkl/norm/warp_softmax.h:120-150 computes it
 * (is_log_softmax = true): max over the row, sum of exp(x - max) in fp32,
 * dst = x - max - log(sum).  Sequential sum order (the device kernel's
 * order is a shuffle tree; results agree to fp32 rounding). */
void pmkl_oracle_log_softmax_fwd_f32(float *dst, const float *src, int elements,
                                     int stride, int rows) {
    for (int b = 0; b < rows; b++) {
        const float *src_b = src + (int64_t)b * stride;
        float *dst_b = dst + (int64_t)b * stride;
        float max_v = -INFINITY;
        for (int i = 0; i < elements; i++) max_v = src_b[i] > max_v ? src_b[i] : max_v;
        float sum = 0;
        for (int i = 0; i < elements; i++) sum += expf(src_b[i] - max_v);
        const float lse = logf(sum);
        for (int i = 0; i < elements; i++) dst_b[i] = src_b[i] - max_v - lse;
    }
}

/* pmkl_pytorch_ext/fused_self_attention.cpp:66-135
 * (pmkl_cpu::host_self_attention_backward<float>), loop for loop, with the
 * reference's operation order: O(S^3 D).  dq, dk, dv are zeroed first, as
 * at::zeros_like does in fused_self_attention_bw (:186-188).  m, l are the
 * forward's row max and exp-sum, used as given: p = exp(s - m) / l. */
void pmkl_oracle_attention_bwd_exact_f32(const float *dout, const float *q, const float *k,
                                         const float *v, const float *out_m, const float *out_l,
                                         float *dq, float *dk, float *dv, int64_t BH, int S,
                                         int D, int causal) {
    const float neg_inf = -INFINITY;
    const float scale = 1.0f / sqrtf((float)D);
    const size_t n_el = (size_t)BH * (size_t)S * (size_t)D;
    memset(dq, 0, n_el * sizeof(float));
    memset(dk, 0, n_el * sizeof(float));
    memset(dv, 0, n_el * sizeof(float));
    for (int64_t b = 0; b < BH; b++) {
        const int64_t off = b * (int64_t)S * D;
        float *dq_b = dq + off, *dk_b = dk + off, *dv_b = dv + off;
        const float *do_b = dout + off, *q_b = q + off, *k_b = k + off, *v_b = v + off;
        const float *m_b = out_m + b * S, *l_b = out_l + b * S;
        for (int m = 0; m < S; m++) {     /* key row */
            for (int n = 0; n < S; n++) { /* query row */
                float qk = 0;
                for (int kk = 0; kk < D; kk++) qk += q_b[(int64_t)n * D + kk] * k_b[(int64_t)m * D + kk];
                qk = qk * scale;
                if (causal) qk = n >= m ? qk : neg_inf;
                const float p = expf(qk - m_b[n]) / l_b[n];
                for (int kk = 0; kk < D; kk++) dv_b[(int64_t)m * D + kk] += p * do_b[(int64_t)n * D + kk];
                float acc_d = 0;
                for (int im = 0; im < S; im++) {
                    float dqksm = 0;
                    for (int kk = 0; kk < D; kk++) dqksm += do_b[(int64_t)n * D + kk] * v_b[(int64_t)im * D + kk];
                    float d_;
                    if (im == m) {
                        d_ = dqksm * p * (1 - p);
                    } else {
                        float qk_ = 0;
                        for (int kk = 0; kk < D; kk++) qk_ += q_b[(int64_t)n * D + kk] * k_b[(int64_t)im * D + kk];
                        qk_ = qk_ * scale;
                        if (causal) qk_ = n >= im ? qk_ : neg_inf;
                        const float p_ = expf(qk_ - m_b[n]) / l_b[n];
                        d_ = -dqksm * p_ * p;
                    }
                    d_ *= scale;
                    acc_d += d_;
                }
                for (int kk = 0; kk < D; kk++) dq_b[(int64_t)n * D + kk] += acc_d * k_b[(int64_t)m * D + kk];
                for (int kk = 0; kk < D; kk++) dk_b[(int64_t)m * D + kk] += acc_d * q_b[(int64_t)n * D + kk];
            }
        }
    }
}

/* The same gradient in O(S^2 D), with double accumulation: the reference's
 * inner sum over keys (:99-121) equals scale * p_m * (dP_m - sum_j p_j dP_j),
 * dP_j = dout_n . v_j, because its inner_m == m term is dP_m p_m (1 - p_m) and
 * every other term is -dP_j p_j p_m.  Scores and p are formed in float as the
 * reference forms them (:86-91); everything after in double.  Used where the
 * O(S^3 D) form would take too long.  Returns 0, or -1 on allocation failure. */
int pmkl_oracle_attention_bwd_f32(const float *dout, const float *q, const float *k,
                                  const float *v, const float *out_m, const float *out_l,
                                  float *dq, float *dk, float *dv, int64_t BH, int S, int D,
                                  int causal, float scale) {
    if (BH <= 0 || S <= 0 || D <= 0) return 0;
    double *dk_acc = (double *)malloc(sizeof(double) * (size_t)S * D);
    double *dv_acc = (double *)malloc(sizeof(double) * (size_t)S * D);
    double *dq_acc = (double *)malloc(sizeof(double) * (size_t)D);
    float *p = (float *)malloc(sizeof(float) * (size_t)S);
    double *dp = (double *)malloc(sizeof(double) * (size_t)S);
    int rc = 0;
    if (!dk_acc || !dv_acc || !dq_acc || !p || !dp) {
        rc = -1;
        goto done;
    }
    for (int64_t b = 0; b < BH; b++) {
        const int64_t off = b * (int64_t)S * D;
        const float *do_b = dout + off, *q_b = q + off, *k_b = k + off, *v_b = v + off;
        const float *m_b = out_m + b * S, *l_b = out_l + b * S;
        memset(dk_acc, 0, sizeof(double) * (size_t)S * D);
        memset(dv_acc, 0, sizeof(double) * (size_t)S * D);
        for (int n = 0; n < S; n++) {
            const float *q_n = q_b + (int64_t)n * D, *do_n = do_b + (int64_t)n * D;
            double delta = 0.0;
            for (int j = 0; j < S; j++) {
                const float *k_j = k_b + (int64_t)j * D, *v_j = v_b + (int64_t)j * D;
                float qk = 0;
                for (int kk = 0; kk < D; kk++) qk += q_n[kk] * k_j[kk];
                qk = qk * scale;
                if (causal && j > n) qk = -INFINITY;
                p[j] = expf(qk - m_b[n]) / l_b[n];
                double acc = 0.0;
                for (int kk = 0; kk < D; kk++) acc += (double)do_n[kk] * (double)v_j[kk];
                dp[j] = acc;
                delta += (double)p[j] * acc;
            }
            for (int kk = 0; kk < D; kk++) dq_acc[kk] = 0.0;
            for (int j = 0; j < S; j++) {
                if (p[j] == 0.0f) continue;
                const float *k_j = k_b + (int64_t)j * D;
                const double ds = (double)p[j] * (dp[j] - delta) * (double)scale;
                for (int kk = 0; kk < D; kk++) {
                    dq_acc[kk] += ds * (double)k_j[kk];
                    dk_acc[(int64_t)j * D + kk] += ds * (double)q_n[kk];
                    dv_acc[(int64_t)j * D + kk] += (double)p[j] * (double)do_n[kk];
                }
            }
            for (int kk = 0; kk < D; kk++) dq[off + (int64_t)n * D + kk] = (float)dq_acc[kk];
        }
        for (int64_t i = 0; i < (int64_t)S * D; i++) {
            dk[off + i] = (float)dk_acc[i];
            dv[off + i] = (float)dv_acc[i];
        }
    }
done:
    free(dk_acc);
    free(dv_acc);
    free(dq_acc);
    free(p);
    free(dp);
    return rc;
}
