/* TEST INFRASTRUCTURE (oracle) -- not part of the product.
 *
 * CPU restatement, in plain C, of DirkTensor's attention hot path:
 *   QKV projection -> QK-RMSNorm -> RoPE -> causal flash attention -> O projection.
 * Every function cites the reference file:line it follows (paths relative to
 * the DirkTensor source tree).  It is pinned against the reference's own
 * FlashAttention.cpp, compiled in place (oracle/_ref), and against golden
 * vectors produced by that build (tests/golden).  Only tests/, the smoke check
 * and bench.py's CPU-baseline leg may load this library; the product never does.
 *
 * Layouts follow the reference: activations [B,T,H,D] / [B,T,d_model] row-major
 * fp32, weights [out,in] row-major (as in the .npy checkpoint files).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <omp.h>

/* OpenBLAS (scipy's bundled 0.3.x build).  The reference's projections go
 * through xt::linalg::dot, i.e. a CBLAS sgemm (OlmoAttention.cpp:68,74,80,104). */
void scipy_cblas_sgemm(int order, int ta, int tb, int m, int n, int k, float alpha,
                       const float* a, int lda, const float* b, int ldb, float beta,
                       float* c, int ldc);
void scipy_openblas_set_num_threads(int n);

void or_set_threads(int n) {
    if (n <= 0) n = omp_get_num_procs();
    omp_set_num_threads(n);
    scipy_openblas_set_num_threads(n);
}

/* RoPE tables, OlmoAttention.cpp:16-36: inv_freq[i] = 1/theta^(2i/head_dim)
 * in double; angle[p][j] = p * inv_freq[j mod head_dim/2] (the table is the
 * concatenation of freqs with itself); sin/cos evaluated in double, then cast
 * to float.  Outputs: [max_seq, head_dim] each.  Built without fast-math so
 * sin/cos are the scalar libm ones (a vectorised sin may differ by an ulp). */
__attribute__((optimize("no-fast-math"))) void or_rope_tables(int max_seq, int head_dim, double theta, float* sin_out, float* cos_out) {
    const int half = head_dim / 2;
    for (int p = 0; p < max_seq; ++p) {
        for (int j = 0; j < head_dim; ++j) {
            const int i = j % half;
            const double inv_freq = 1.0 / pow(theta, (double)(2 * i) / (double)head_dim);
            const double ang = (double)p * inv_freq;
            sin_out[(size_t)p * head_dim + j] = (float)sin(ang);
            cos_out[(size_t)p * head_dim + j] = (float)cos(ang);
        }
    }
}

/* RMSNorm forward, RMSNorm.cpp:15-22 (eps RMSNorm.h:10): per row of `dim`,
 * rms = sqrt(sum(x^2)/dim + eps); y = x / rms * g.  fp32 throughout. */
void or_rmsnorm(const float* x, const float* g, float* y, long rows, int dim, float eps) {
#pragma omp parallel for schedule(static)
    for (long r = 0; r < rows; ++r) {
        const float* xr = x + (size_t)r * dim;
        float* yr = y + (size_t)r * dim;
        float ss = 0.0f;
        for (int i = 0; i < dim; ++i) ss += xr[i] * xr[i];
        const float rms = sqrtf(ss / (float)dim + eps);
        for (int i = 0; i < dim; ++i) yr[i] = xr[i] / rms * g[i];
    }
}

/* Rotate-half RoPE, OlmoAttention.cpp:111-146: position = t (no offset);
 * out[d] = x[d]*cos[t][d] - x[d+half]*sin[t][d];
 * out[d+half] = x[d+half]*cos[t][d+half] + x[d]*sin[t][d+half]. */
void or_rope(const float* x, float* y, long B, long T, int H, int D,
             const float* sin_t, const float* cos_t) {
    const int half = D / 2;
#pragma omp parallel for collapse(2) schedule(static)
    for (long b = 0; b < B; ++b) {
        for (long t = 0; t < T; ++t) {
            for (int h = 0; h < H; ++h) {
                const size_t base = (((size_t)b * T + t) * H + h) * D;
                const float* c = cos_t + (size_t)t * D;
                const float* s = sin_t + (size_t)t * D;
                for (int d = 0; d < half; ++d)
                    y[base + d] = x[base + d] * c[d] - x[base + d + half] * s[d];
                for (int d = 0; d < half; ++d)
                    y[base + d + half] = x[base + d + half] * c[d + half] + x[base + d] * s[d + half];
            }
        }
    }
}

/* y[M,N] = x[M,K] . w[N,K]^T  (xt::linalg::dot(x, transpose(W)),
 * OlmoAttention.cpp:68,74,80,103-105), through CBLAS sgemm. */
void or_linear(const float* x, const float* w, float* y, long M, int N, int K) {
    scipy_cblas_sgemm(101 /*RowMajor*/, 111 /*NoTrans*/, 112 /*Trans*/, (int)M, N, K, 1.0f,
                      x, K, w, K, 0.0f, y, N);
}

/* Causal tiled online-softmax attention, FlashAttention.cpp:24-182.
 * Same blocking (Br = Bc = 256, :21-22), same block skip rule
 * (skip iff causal && q_start < k_start, :76), same element mask
 * (masked iff q_pos < k_pos, :102), same per-block update order
 * (local max, P = exp(s - m_local), l_local, PV, then
 *  m_new = max(m, m_local), alpha = exp(m - m_new), beta = exp(m_local - m_new),
 *  l = l*alpha + l_local*beta, O = O*alpha + PV*beta, :134-156), final O/l or 0
 * when l == 0 (:159-176).  softmax_m / softmax_l are the final m and l per row
 * (m in units of the scaled score).  Dot products are plain fp32 loops. */
#define OR_BLK 256
void or_flash_fwd(const float* Q, const float* K, const float* V, float* O, float* Mo, float* Lo,
                  long B, long T, int H, int D, float scale, int causal) {
    const size_t rs = (size_t)H * D; /* token row stride */
#pragma omp parallel
    {
        float* S = (float*)malloc(sizeof(float) * OR_BLK * OR_BLK);
        float* PV = (float*)malloc(sizeof(float) * OR_BLK * D);
        float* Oacc = (float*)malloc(sizeof(float) * OR_BLK * D);
        float m[OR_BLK], l[OR_BLK], ml[OR_BLK], ll[OR_BLK];
#pragma omp for schedule(dynamic, 1)
        for (long bh = 0; bh < B * H; ++bh) {
            const long b = bh / H;
            const int h = (int)(bh % H);
            const float* q0 = Q + (size_t)b * T * rs + (size_t)h * D;
            const float* k0 = K + (size_t)b * T * rs + (size_t)h * D;
            const float* v0 = V + (size_t)b * T * rs + (size_t)h * D;
            for (long qs = 0; qs < T; qs += OR_BLK) {
                const long br = (T - qs < OR_BLK) ? T - qs : OR_BLK;
                for (long i = 0; i < br; ++i) { m[i] = -INFINITY; l[i] = 0.0f; }
                memset(Oacc, 0, sizeof(float) * br * D);
                for (long ks = 0; ks < T; ks += OR_BLK) {
                    const long bc = (T - ks < OR_BLK) ? T - ks : OR_BLK;
                    if (causal && qs < ks) continue;
                    for (long i = 0; i < br; ++i) {
                        const float* qi = q0 + (size_t)(qs + i) * rs;
                        for (long j = 0; j < bc; ++j) {
                            const float* kj = k0 + (size_t)(ks + j) * rs;
                            float acc = 0.0f;
                            for (int d = 0; d < D; ++d) acc += qi[d] * kj[d];
                            S[i * OR_BLK + j] = scale * acc;
                        }
                    }
                    for (long i = 0; i < br; ++i) {
                        float mx = -INFINITY;
                        for (long j = 0; j < bc; ++j) {
                            if (causal && qs + i < ks + j) S[i * OR_BLK + j] = -INFINITY;
                            else if (S[i * OR_BLK + j] > mx) mx = S[i * OR_BLK + j];
                        }
                        ml[i] = mx;
                        float sum = 0.0f;
                        for (long j = 0; j < bc; ++j) {
                            const float s = S[i * OR_BLK + j];
                            const float p = (s > -INFINITY) ? expf(s - mx) : 0.0f;
                            S[i * OR_BLK + j] = p; /* S now holds P */
                            sum += p;
                        }
                        ll[i] = sum;
                    }
                    for (long i = 0; i < br; ++i) {
                        float* pv = PV + i * D;
                        for (int d = 0; d < D; ++d) pv[d] = 0.0f;
                        for (long j = 0; j < bc; ++j) {
                            const float p = S[i * OR_BLK + j];
                            const float* vj = v0 + (size_t)(ks + j) * rs;
                            for (int d = 0; d < D; ++d) pv[d] += p * vj[d];
                        }
                    }
                    for (long i = 0; i < br; ++i) {
                        const float mn = (m[i] > ml[i]) ? m[i] : ml[i];
                        const float alpha = (m[i] > -INFINITY) ? expf(m[i] - mn) : 0.0f;
                        const float beta = (ml[i] > -INFINITY) ? expf(ml[i] - mn) : 0.0f;
                        l[i] = l[i] * alpha + ll[i] * beta;
                        for (int d = 0; d < D; ++d) Oacc[i * D + d] = Oacc[i * D + d] * alpha + PV[i * D + d] * beta;
                        m[i] = mn;
                    }
                }
                for (long i = 0; i < br; ++i) {
                    const size_t row = ((size_t)b * T + qs + i) * H + h;
                    if (Mo) Mo[row] = m[i];
                    if (Lo) Lo[row] = l[i];
                    for (int d = 0; d < D; ++d) O[row * D + d] = (l[i] > 0.0f) ? Oacc[i * D + d] / l[i] : 0.0f;
                }
            }
        }
        free(S); free(PV); free(Oacc);
    }
}

/* fp64 "truth" for selected rows: direct softmax over keys 0..t (causal) or
 * 0..T-1, all in double.  rows: n triples (b, t, h).  out: [n, D];
 * m_out/l_out: [n] with the reference's meaning (m = max scaled score,
 * l = sum exp(s - m)).  Used to calibrate tolerances and for size-independent
 * spot checks at full sizes. */
void or_attention_rows_f64(const float* Q, const float* K, const float* V, long B, long T, int H, int D,
                           double scale, int causal, const long* rows, long n,
                           double* out, double* m_out, double* l_out) {
    const size_t rs = (size_t)H * D;
#pragma omp parallel
    {
        double* s = (double*)malloc(sizeof(double) * (size_t)T);
#pragma omp for schedule(dynamic, 4)
        for (long r = 0; r < n; ++r) {
            const long b = rows[3 * r + 0], t = rows[3 * r + 1], h = rows[3 * r + 2];
            const float* qi = Q + ((size_t)b * T + t) * rs + (size_t)h * D;
            const long kend = causal ? t + 1 : T;
            double mx = -INFINITY;
            for (long j = 0; j < kend; ++j) {
                const float* kj = K + ((size_t)b * T + j) * rs + (size_t)h * D;
                double acc = 0.0;
                for (int d = 0; d < D; ++d) acc += (double)qi[d] * (double)kj[d];
                s[j] = acc * scale;
                if (s[j] > mx) mx = s[j];
            }
            double sum = 0.0;
            for (long j = 0; j < kend; ++j) { s[j] = exp(s[j] - mx); sum += s[j]; }
            double* o = out + (size_t)r * D;
            for (int d = 0; d < D; ++d) o[d] = 0.0;
            for (long j = 0; j < kend; ++j) {
                const float* vj = V + ((size_t)b * T + j) * rs + (size_t)h * D;
                for (int d = 0; d < D; ++d) o[d] += s[j] * (double)vj[d];
            }
            for (int d = 0; d < D; ++d) o[d] /= sum;
            if (m_out) m_out[r] = mx;
            if (l_out) l_out[r] = sum;
        }
        free(s);
    }
}

/* One attention layer, OlmoAttention::forward (OlmoAttention.cpp:56-108):
 * q = rope(qnorm(x Wq^T)), k = rope(knorm(x Wk^T)), v = x Wv^T,
 * a = flash(q, k, v, 1/sqrt(head_dim), causal), y = a Wo^T.
 * x: [B,T,d]; W*: [d,d]; qg,kg: [d]; y: [B,T,d].  Optional intermediates
 * (q_out, k_out, v_out, a_out: [B,T,d], pass NULL to skip) are the tensors the
 * GPU prologue and flash kernels produce, for stage-wise comparisons. */
void or_attention_layer(const float* x, const float* wq, const float* wk, const float* wv,
                        const float* wo, const float* qg, const float* kg, float* y,
                        long B, long T, int d_model, int n_heads, float eps, double theta,
                        float* q_out, float* k_out, float* v_out, float* a_out) {
    const long M = B * T;
    const int D = d_model / n_heads;
    const size_t n = (size_t)M * d_model;
    float* p = (float*)malloc(sizeof(float) * n);
    float* q = (float*)malloc(sizeof(float) * n);
    float* k = (float*)malloc(sizeof(float) * n);
    float* v = (float*)malloc(sizeof(float) * n);
    float* a = (float*)malloc(sizeof(float) * n);
    float* st = (float*)malloc(sizeof(float) * (size_t)T * D);
    float* ct = (float*)malloc(sizeof(float) * (size_t)T * D);
    or_rope_tables((int)T, D, theta, st, ct);

    or_linear(x, wq, p, M, d_model, d_model);
    or_rmsnorm(p, qg, a, M, d_model, eps);
    or_rope(a, q, B, T, n_heads, D, st, ct);

    or_linear(x, wk, p, M, d_model, d_model);
    or_rmsnorm(p, kg, a, M, d_model, eps);
    or_rope(a, k, B, T, n_heads, D, st, ct);

    or_linear(x, wv, v, M, d_model, d_model);

    or_flash_fwd(q, k, v, a, NULL, NULL, B, T, n_heads, D, 1.0f / sqrtf((float)D), 1);
    or_linear(a, wo, y, M, d_model, d_model);

    if (q_out) memcpy(q_out, q, sizeof(float) * n);
    if (k_out) memcpy(k_out, k, sizeof(float) * n);
    if (v_out) memcpy(v_out, v, sizeof(float) * n);
    if (a_out) memcpy(a_out, a, sizeof(float) * n);
    free(p); free(q); free(k); free(v); free(a); free(st); free(ct);
}

/* SwiGLU MLP, OlmoMlp.cpp:26-63: up = x Wup^T, gate = x Wgate^T (weights
 * [hidden, d]), act = gate / (1 + exp(-gate)) * up (:48-52), out = act Wdown^T
 * (Wdown [d, hidden]).  x, out: [M, d]. */
void or_mlp(const float* x, const float* w_gate, const float* w_up, const float* w_down, float* out,
            long M, int d, int hidden) {
    float* up = (float*)malloc(sizeof(float) * (size_t)M * hidden);
    float* gate = (float*)malloc(sizeof(float) * (size_t)M * hidden);
    or_linear(x, w_up, up, M, hidden, d);
    or_linear(x, w_gate, gate, M, hidden, d);
#pragma omp parallel for schedule(static)
    for (long i = 0; i < M * (long)hidden; ++i) {
        const float g = gate[i];
        gate[i] = g / (1.0f + expf(-g)) * up[i];
    }
    or_linear(gate, w_down, out, M, d, hidden);
    free(up);
    free(gate);
}

/* Weights of one decoder layer, in the checkpoint's layouts. */
typedef struct {
    const float *q_proj, *k_proj, *v_proj, *o_proj, *q_norm, *k_norm;
    const float *post_attention_norm, *gate_proj, *up_proj, *down_proj, *post_feedforward_norm;
} or_layer_weights;

/* Full model prefill, OlmoModel.cpp:25-48 with OlmoBlock.cpp:13-21:
 * x = embed[ids]; per layer: h = x + norm_pa(attn(x)); x = h + norm_pf(mlp(h));
 * logits = norm_final(x) Wlm^T.  ids: [B, T] uint32; logits: [B, T, vocab].
 * n_layers and vocab are parameters (the reference fixes 16 and 100352) so
 * tests can run reduced models; everything else follows the reference. */
void or_model_forward(const unsigned* ids, long B, long T, const float* embed, const or_layer_weights* layers,
                      int n_layers, const float* final_norm, const float* lm_head, int vocab, int d_model,
                      int n_heads, int hidden, float eps, double theta, float* logits) {
    const long M = B * T;
    const size_t n = (size_t)M * d_model;
    float* x = (float*)malloc(sizeof(float) * n);
    float* y = (float*)malloc(sizeof(float) * n);
    float* t = (float*)malloc(sizeof(float) * n);
    for (long i = 0; i < M; ++i) memcpy(x + (size_t)i * d_model, embed + (size_t)ids[i] * d_model, sizeof(float) * d_model);
    for (int li = 0; li < n_layers; ++li) {
        const or_layer_weights* w = &layers[li];
        or_attention_layer(x, w->q_proj, w->k_proj, w->v_proj, w->o_proj, w->q_norm, w->k_norm, y, B, T, d_model,
                           n_heads, eps, theta, NULL, NULL, NULL, NULL);
        or_rmsnorm(y, w->post_attention_norm, t, M, d_model, eps);
        for (size_t i = 0; i < n; ++i) x[i] += t[i]; /* x is now h */
        or_mlp(x, w->gate_proj, w->up_proj, w->down_proj, y, M, d_model, hidden);
        or_rmsnorm(y, w->post_feedforward_norm, t, M, d_model, eps);
        for (size_t i = 0; i < n; ++i) x[i] += t[i];
    }
    or_rmsnorm(x, final_norm, t, M, d_model, eps);
    or_linear(t, lm_head, logits, M, vocab, d_model);
    free(x);
    free(y);
    free(t);
}

/* ------------------------------------------------------------------------
 * Training path (backward) restatements.
 * ------------------------------------------------------------------------ */

/* Generic row-major CBLAS sgemm, the form of every projection-gradient call in
 * OlmoAttention::backward (OlmoAttention.cpp:201-205, 240-267, 278-298). */
void or_sgemm(int trans_a, int trans_b, int M, int N, int K, float alpha, const float* A, int lda,
              const float* Bm, int ldb, float beta, float* C, int ldc) {
    scipy_cblas_sgemm(101, trans_a ? 112 : 111, trans_b ? 112 : 111, M, N, K, alpha, A, lda, Bm, ldb, beta, C,
                      ldc);
}

/* RMSNorm forward that also returns the per-row rms (RMSNorm.cpp:15-22, the
 * m_act_rms member the backward divides by). */
void or_rmsnorm_rms(const float* x, const float* g, float* y, float* rms_out, long rows, int dim, float eps) {
#pragma omp parallel for schedule(static)
    for (long r = 0; r < rows; ++r) {
        const float* xr = x + (size_t)r * dim;
        float* yr = y + (size_t)r * dim;
        float ss = 0.0f;
        for (int i = 0; i < dim; ++i) ss += xr[i] * xr[i];
        const float rms = sqrtf(ss / (float)dim + eps);
        rms_out[r] = rms;
        for (int i = 0; i < dim; ++i) yr[i] = xr[i] / rms * g[i];
    }
}

/* RMSNorm backward, RMSNorm.cpp:24-36, with y = the forward output (x/rms*g):
 *   c = mean(dy * y) over the row;  x_hat = y / g (recomputed, :30);
 *   dg += sum over rows of dy * x_hat (:31);  dx = (g*dy - x_hat*c) / rms (:35). */
void or_rmsnorm_bwd(const float* dy, const float* y, const float* g, const float* rms, float* dx, float* dg,
                    long rows, int dim) {
#pragma omp parallel for schedule(static)
    for (long r = 0; r < rows; ++r) {
        const float* dyr = dy + (size_t)r * dim;
        const float* yr = y + (size_t)r * dim;
        float* dxr = dx + (size_t)r * dim;
        float c = 0.0f;
        for (int i = 0; i < dim; ++i) c += dyr[i] * yr[i];
        c /= (float)dim;
        for (int i = 0; i < dim; ++i) {
            const float xh = yr[i] / g[i];
            dxr[i] = (g[i] * dyr[i] - xh * c) / rms[r];
        }
    }
    /* weight gradient: column sums in row order */
#pragma omp parallel for schedule(static)
    for (int i = 0; i < dim; ++i) {
        float acc = 0.0f;
        for (long r = 0; r < rows; ++r) acc += dy[(size_t)r * dim + i] * (y[(size_t)r * dim + i] / g[i]);
        dg[i] += acc;
    }
}

/* RoPE backward, OlmoAttention.cpp:149-187 (the transpose of the rotation):
 *   d_in[d]      =  d_out[d]*cos[t][d] + d_out[d+half]*sin[t][d+half]
 *   d_in[d+half] = -d_out[d]*sin[t][d] + d_out[d+half]*cos[t][d+half]. */
void or_rope_bwd(const float* dy, float* dx, long B, long T, int H, int D, const float* sin_t,
                 const float* cos_t) {
    const int half = D / 2;
#pragma omp parallel for collapse(2) schedule(static)
    for (long b = 0; b < B; ++b) {
        for (long t = 0; t < T; ++t) {
            for (int h = 0; h < H; ++h) {
                const size_t base = (((size_t)b * T + t) * H + h) * D;
                const float* c = cos_t + (size_t)t * D;
                const float* s = sin_t + (size_t)t * D;
                for (int d = 0; d < half; ++d) {
                    dx[base + d] = dy[base + d] * c[d] + dy[base + d + half] * s[d + half];
                    dx[base + d + half] = -dy[base + d] * s[d] + dy[base + d + half] * c[d + half];
                }
            }
        }
    }
}

/* Flash attention backward, FlashAttention.cpp:185-359.  Same blocking
 * (256 x 256), same skip rule (causal && q_start < k_start, :247), per Q
 * block: D[i] = O[i].dO[i] (:232-237); per K block: S = scale * Q K^T (:250),
 * P = exp(s - m)/l or 0 where q_pos < k_pos (:262-275), dP = dO V^T (:278),
 * dS = P * (dP - D) * scale (:290-296), dV += P^T dO (:299-314),
 * dQ_block += dS K (:317-325), dK += dS^T Q (:328-343); dQ written per Q
 * block (:347-351).  Dot products are plain fp32 loops in index order. */
void or_flash_bwd(const float* dO, const float* O, const float* Mi, const float* Li, const float* Q,
                  const float* K, const float* V, float* dQ, float* dK, float* dV, long B, long T, int H, int D,
                  float scale, int causal) {
    const size_t rs = (size_t)H * D;
    const size_t nall = (size_t)B * T * H * D;
    memset(dQ, 0, nall * sizeof(float));
    memset(dK, 0, nall * sizeof(float));
    memset(dV, 0, nall * sizeof(float));
#pragma omp parallel
    {
        float* P = (float*)malloc(sizeof(float) * OR_BLK * OR_BLK);
        float* dS = (float*)malloc(sizeof(float) * OR_BLK * OR_BLK);
        float* Dr = (float*)malloc(sizeof(float) * OR_BLK);
        float* dQb = (float*)malloc(sizeof(float) * OR_BLK * D);
#pragma omp for schedule(dynamic, 1)
        for (long bh = 0; bh < B * H; ++bh) {
            const long b = bh / H;
            const int h = (int)(bh % H);
            for (long q0 = 0; q0 < T; q0 += OR_BLK) {
                const long Br = (T - q0) < OR_BLK ? (T - q0) : OR_BLK;
                for (long i = 0; i < Br; ++i) {
                    const size_t ro = ((size_t)b * T + q0 + i) * rs + (size_t)h * D;
                    float acc = 0.0f;
                    for (int d = 0; d < D; ++d) acc += O[ro + d] * dO[ro + d];
                    Dr[i] = acc;
                }
                memset(dQb, 0, sizeof(float) * Br * D);
                for (long k0 = 0; k0 < T; k0 += OR_BLK) {
                    const long Bc = (T - k0) < OR_BLK ? (T - k0) : OR_BLK;
                    if (causal && q0 < k0) continue;
                    for (long i = 0; i < Br; ++i) {
                        const size_t rq = ((size_t)b * T + q0 + i) * rs + (size_t)h * D;
                        const size_t ist = ((size_t)b * T + q0 + i) * H + h;
                        const float m = Mi[ist], l = Li[ist], Di = Dr[i];
                        for (long j = 0; j < Bc; ++j) {
                            const size_t rk = ((size_t)b * T + k0 + j) * rs + (size_t)h * D;
                            float p = 0.0f, dp = 0.0f;
                            if (!(causal && q0 + i < k0 + j)) {
                                float s = 0.0f;
                                for (int d = 0; d < D; ++d) s += Q[rq + d] * K[rk + d];
                                p = expf(scale * s - m) / l;
                            }
                            for (int d = 0; d < D; ++d) dp += dO[rq + d] * V[rk + d];
                            P[i * OR_BLK + j] = p;
                            dS[i * OR_BLK + j] = p * (dp - Di) * scale;
                        }
                    }
                    for (long j = 0; j < Bc; ++j) {
                        const size_t rk = ((size_t)b * T + k0 + j) * rs + (size_t)h * D;
                        for (int d = 0; d < D; ++d) {
                            float av = 0.0f, ak = 0.0f;
                            for (long i = 0; i < Br; ++i) {
                                const size_t rq = ((size_t)b * T + q0 + i) * rs + (size_t)h * D;
                                av += P[i * OR_BLK + j] * dO[rq + d];
                                ak += dS[i * OR_BLK + j] * Q[rq + d];
                            }
                            dV[rk + d] += av;
                            dK[rk + d] += ak;
                        }
                    }
                    for (long i = 0; i < Br; ++i) {
                        for (int d = 0; d < D; ++d) {
                            float acc = 0.0f;
                            for (long j = 0; j < Bc; ++j) {
                                const size_t rk = ((size_t)b * T + k0 + j) * rs + (size_t)h * D;
                                acc += dS[i * OR_BLK + j] * K[rk + d];
                            }
                            dQb[i * D + d] += acc;
                        }
                    }
                }
                for (long i = 0; i < Br; ++i) {
                    const size_t rq = ((size_t)b * T + q0 + i) * rs + (size_t)h * D;
                    for (int d = 0; d < D; ++d) dQ[rq + d] = dQb[i * D + d];
                }
            }
        }
        free(P);
        free(dS);
        free(Dr);
        free(dQb);
    }
}
