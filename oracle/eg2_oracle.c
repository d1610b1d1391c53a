/*
 * CPU oracle for the EmbeddingGemma 2 hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's CPU f32 path, used by tests/, by
 * __graft_entry__.smoke() and by bench.py's cpu_baseline leg as the checker and the timed
 * CPU baseline. It is never linked into, or called by, the CUDA library.
 *
 * Followed line by line (paths inside the reference project):
 *   text forward     src/text.rs:136-235, embedding scale src/text.rs:53-64
 *   RMSNorm          src/ops.rs:211-238 (f64 sum of squares, (ms as f32 + eps)^-0.5)
 *   GELU (tanh)      src/ops.rs:241-246
 *   softmax          src/ops.rs:270-286
 *   RoPE             src/ops.rs:293-338 (f32 powf inverse frequencies, duplicated halves)
 *   attention        src/ops.rs:364-444 (scale 1, inclusive window, 128-query blocks)
 *   mean / L2        src/ops.rs:451-467 (f64), Matryoshka src/model.rs:677-688
 *   vision tower     src/vision.rs:73-170, :223-293
 * The reference's CPU GEMM is the third-party `gemm` crate 0.19.0 (Cargo.lock), not vendored;
 * sgemm_nt below is this file's own blocked f32 GEMM. Any f32 summation order stays inside
 * the reference's float32 profile.
 *
 * Build: oracle/Makefile (gcc -O3 -mavx2 -mfma -fopenmp -ffp-contract=off). Contraction is
 * off so every elementwise step rounds like the Rust code; the GEMM uses explicit FMAs.
 */
#include <immintrin.h>
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------------------------ */
/* GEMM                                                                                        */
/* ------------------------------------------------------------------------------------------ */

static inline float hsum256(__m256 v) {
    __m128 lo = _mm256_castps256_ps128(v), hi = _mm256_extractf128_ps(v, 1);
    lo = _mm_add_ps(lo, hi);
    __m128 sh = _mm_movehdup_ps(lo);
    lo = _mm_add_ps(lo, sh);
    sh = _mm_movehl_ps(sh, lo);
    lo = _mm_add_ss(lo, sh);
    return _mm_cvtss_f32(lo);
}

/* c[i*ldc + j] = sum_k a[i*lda + k] * b[j*ldb + k] for a block of rows [i0, i1) and all j. */
static void sgemm_nt_rows(int i0, int i1, int n, int k, const float* a, long lda, const float* b, long ldb,
                          float* c, long ldc) {
    const int JB = 64;
    for (int jb = 0; jb < n; jb += JB) {
        int je = jb + JB < n ? jb + JB : n;
        int i = i0;
        for (; i + 4 <= i1; i += 4) {
            int j = jb;
            for (; j + 4 <= je; j += 4) {
                __m256 acc[4][4];
                for (int r = 0; r < 4; r++)
                    for (int s = 0; s < 4; s++) acc[r][s] = _mm256_setzero_ps();
                int kk = 0;
                for (; kk + 8 <= k; kk += 8) {
                    __m256 av[4], bv[4];
                    for (int r = 0; r < 4; r++) av[r] = _mm256_loadu_ps(a + (long)(i + r) * lda + kk);
                    for (int s = 0; s < 4; s++) bv[s] = _mm256_loadu_ps(b + (long)(j + s) * ldb + kk);
                    for (int r = 0; r < 4; r++)
                        for (int s = 0; s < 4; s++) acc[r][s] = _mm256_fmadd_ps(av[r], bv[s], acc[r][s]);
                }
                for (int r = 0; r < 4; r++)
                    for (int s = 0; s < 4; s++) {
                        float t = hsum256(acc[r][s]);
                        for (int q = kk; q < k; q++) t += a[(long)(i + r) * lda + q] * b[(long)(j + s) * ldb + q];
                        c[(long)(i + r) * ldc + j + s] = t;
                    }
            }
            for (; j < je; j++)
                for (int r = 0; r < 4; r++) {
                    __m256 acc = _mm256_setzero_ps();
                    int kk = 0;
                    for (; kk + 8 <= k; kk += 8)
                        acc = _mm256_fmadd_ps(_mm256_loadu_ps(a + (long)(i + r) * lda + kk),
                                              _mm256_loadu_ps(b + (long)j * ldb + kk), acc);
                    float t = hsum256(acc);
                    for (; kk < k; kk++) t += a[(long)(i + r) * lda + kk] * b[(long)j * ldb + kk];
                    c[(long)(i + r) * ldc + j] = t;
                }
        }
        for (; i < i1; i++)
            for (int j = jb; j < je; j++) {
                __m256 acc = _mm256_setzero_ps();
                int kk = 0;
                for (; kk + 8 <= k; kk += 8)
                    acc = _mm256_fmadd_ps(_mm256_loadu_ps(a + (long)i * lda + kk), _mm256_loadu_ps(b + (long)j * ldb + kk),
                                          acc);
                float t = hsum256(acc);
                for (; kk < k; kk++) t += a[(long)i * lda + kk] * b[(long)j * ldb + kk];
                c[(long)i * ldc + j] = t;
            }
    }
}

/* Serial NT GEMM with strides (used inside already-parallel attention tasks). */
static void sgemm_nt_serial(int m, int n, int k, const float* a, long lda, const float* b, long ldb, float* c, long ldc) {
    if (m == 0 || n == 0) return;
    sgemm_nt_rows(0, m, n, k, a, lda, b, ldb, c, ldc);
}

/* out[m x n] = x[m x k] . w[n x k]^T  (src/ops.rs:131-137), parallel over row blocks. */
void eg2o_sgemm_nt(int m, int n, int k, const float* x, const float* w, float* out) {
    if (m <= 0 || n <= 0) return;
    const int RB = 16;
    int nblk = (m + RB - 1) / RB;
    if (nblk >= 2 * omp_get_max_threads() || n < 256) {
#pragma omp parallel for schedule(dynamic, 1)
        for (int b = 0; b < nblk; b++) {
            int i0 = b * RB, i1 = i0 + RB < m ? i0 + RB : m;
            sgemm_nt_rows(i0, i1, n, k, x, k, w, k, out, n);
        }
    } else {
        /* Few rows: split the output columns instead. */
        const int CB = 64;
        int ncb = (n + CB - 1) / CB;
#pragma omp parallel for schedule(dynamic, 1)
        for (int cb = 0; cb < ncb; cb++) {
            int j0 = cb * CB, j1 = j0 + CB < n ? j0 + CB : n;
            sgemm_nt_rows(0, m, j1 - j0, k, x, k, w + (long)j0 * k, k, out + j0, n);
        }
    }
}

/* ------------------------------------------------------------------------------------------ */
/* Norms, activations, RoPE                                                                    */
/* ------------------------------------------------------------------------------------------ */

/* src/ops.rs:211-238 */
static void rms_norm_row(float* row, int dim, const float* w, float eps) {
    double ss = 0.0;
    for (int i = 0; i < dim; i++) ss += (double)row[i] * (double)row[i];
    float ms = (float)(ss / (double)dim) + eps;
    float inv = powf(ms, -0.5f);
    if (w)
        for (int i = 0; i < dim; i++) row[i] = row[i] * inv * w[i];
    else
        for (int i = 0; i < dim; i++) row[i] *= inv;
}

void eg2o_rms_norm(float* x, long rows, int dim, const float* w, float eps) {
#pragma omp parallel for schedule(static) if (rows * dim >= (1 << 15))
    for (long r = 0; r < rows; r++) rms_norm_row(x + r * dim, dim, w, eps);
}

/* src/ops.rs:241-246 */
static inline float gelu_tanh(float x) {
    const float BETA = 0.79788456f, KAPPA = 0.044715f;
    float inner = BETA * (x + KAPPA * x * x * x);
    return 0.5f * x * (1.0f + tanhf(inner));
}

float eg2o_gelu_tanh(float x) { return gelu_tanh(x); }

/* src/ops.rs:293-295 */
static void rope_inv_freq(double base, int dim, float* inv) {
    for (int i = 0; i < dim / 2; i++) inv[i] = 1.0f / powf((float)base, (float)(2 * i) / (float)dim);
}

/* src/ops.rs:319-326 */
static inline void rope_apply(float* x, int len, const float* c, const float* s) {
    int half = len / 2;
    for (int i = 0; i < half; i++) {
        float x1 = x[i], x2 = x[half + i];
        x[i] = x1 * c[i] - x2 * s[i];
        x[half + i] = x2 * c[half + i] + x1 * s[half + i];
    }
}

/* cos/sin [n_pos, hd] with duplicated halves (src/ops.rs:298-314). */
static void rope_tables(const float* positions, long n, const float* inv, int half, float* cs, float* sn) {
    int dim = 2 * half;
#pragma omp parallel for schedule(static) if (n >= 1024)
    for (long t = 0; t < n; t++)
        for (int i = 0; i < half; i++) {
            float f = positions[t] * inv[i];
            float s = sinf(f), c = cosf(f);
            cs[t * dim + i] = c;
            cs[t * dim + half + i] = c;
            sn[t * dim + i] = s;
            sn[t * dim + half + i] = s;
        }
}

/* src/ops.rs:270-286 */
static void softmax_row(float* row, int n) {
    float mx = -INFINITY;
    for (int i = 0; i < n; i++)
        if (row[i] > mx) mx = row[i];
    float sum = 0.f;
    for (int i = 0; i < n; i++) {
        row[i] = expf(row[i] - mx);
        sum += row[i];
    }
    float inv = 1.0f / sum;
    for (int i = 0; i < n; i++) row[i] *= inv;
}

/* ------------------------------------------------------------------------------------------ */
/* Attention (src/ops.rs:364-444): one sequence, bidirectional, scale 1.                       */
/* window < 0 means global.                                                                    */
/* ------------------------------------------------------------------------------------------ */

#define Q_BLOCK 128

static void attention_task(const float* q, const float* k, const float* v, int seq, int nh, int nkv, int hd, int window,
                           float scale, float* out, int h, int blk, float* scores) {
    int qs = nh * hd, kvs = nkv * hd, group = nh / nkv, g = h / group;
    int q0 = blk * Q_BLOCK, q1 = q0 + Q_BLOCK < seq ? q0 + Q_BLOCK : seq;
    int k0 = 0, k1 = seq;
    if (window >= 0) {
        k0 = q0 > window ? q0 - window : 0;
        k1 = q1 - 1 + window + 1 < seq ? q1 - 1 + window + 1 : seq;
    }
    int qb = q1 - q0, kb = k1 - k0;
    sgemm_nt_serial(qb, kb, hd, q + (long)q0 * qs + (long)h * hd, qs, k + (long)k0 * kvs + (long)g * hd, kvs, scores, kb);
    for (int i = 0; i < qb; i++) {
        int qi = q0 + i;
        float* row = scores + (long)i * kb;
        if (scale != 1.0f)
            for (int jj = 0; jj < kb; jj++) row[jj] *= scale;
        if (window >= 0) {
            int lo = qi > window ? qi - window : 0;
            int hi = qi + window + 1 < seq ? qi + window + 1 : seq;
            for (int jj = 0; jj < kb; jj++) {
                int j = k0 + jj;
                if (j < lo || j >= hi) row[jj] = -INFINITY;
            }
        }
        softmax_row(row, kb);
    }
    /* out[q0.., h] = scores[qb x kb] . v[k0.., g][kb x hd]  (sgemm_nn) */
    for (int i = 0; i < qb; i++) {
        float* o = out + (long)(q0 + i) * qs + (long)h * hd;
        for (int d = 0; d < hd; d++) o[d] = 0.f;
        const float* srow = scores + (long)i * kb;
        for (int jj = 0; jj < kb; jj++) {
            float p = srow[jj];
            const float* vr = v + (long)(k0 + jj) * kvs + (long)g * hd;
            for (int d = 0; d < hd; d++) o[d] += p * vr[d];
        }
    }
}

/* Block-diagonal attention over sequences packed back to back. */
void eg2o_attention_packed(const float* q, const float* k, const float* v, const int64_t* lens, int n_seq, int nh, int nkv,
                           int hd, int window, float* out) {
    int qs = nh * hd, kvs = nkv * hd;
    long* offs = (long*)malloc(sizeof(long) * (n_seq + 1));
    long ntask = 0;
    offs[0] = 0;
    for (int s = 0; s < n_seq; s++) offs[s + 1] = offs[s] + lens[s];
    long* task_start = (long*)malloc(sizeof(long) * (n_seq + 1));
    task_start[0] = 0;
    for (int s = 0; s < n_seq; s++) {
        long nb = (lens[s] + Q_BLOCK - 1) / Q_BLOCK;
        task_start[s + 1] = task_start[s] + nb * nh;
    }
    ntask = task_start[n_seq];
#pragma omp parallel
    {
        float* scores = NULL;
        size_t cap = 0;
#pragma omp for schedule(dynamic, 1)
        for (long t = 0; t < ntask; t++) {
            int s = 0;
            while (task_start[s + 1] <= t) s++;
            long local = t - task_start[s];
            int seq = (int)lens[s];
            int nb = (seq + Q_BLOCK - 1) / Q_BLOCK;
            int h = (int)(local / nb), blk = (int)(local % nb);
            int kbmax = window >= 0 ? (Q_BLOCK + 2 * window < seq ? Q_BLOCK + 2 * window : seq) : seq;
            size_t need = (size_t)Q_BLOCK * (size_t)kbmax;
            if (need > cap) {
                free(scores);
                scores = (float*)malloc(sizeof(float) * need);
                cap = need;
            }
            attention_task(q + offs[s] * qs, k + offs[s] * kvs, v + offs[s] * kvs, seq, nh, nkv, hd, window, 1.0f,
                           out + offs[s] * qs, h, blk, scores);
        }
        free(scores);
    }
    free(task_start);
    free(offs);
}

/* ------------------------------------------------------------------------------------------ */
/* Text backbone (src/text.rs:136-235)                                                         */
/* ------------------------------------------------------------------------------------------ */

typedef struct {
    int hidden, ple_dim, n_layers, n_heads, emb_dim, inter, window;
    float eps;
    const int* head_dim;
    const int* n_kv;
    const int* sliding;
    const double* theta;
    const float* layer_scalar;
    const float* const* input_ln;
    const float* const* post_attn_ln;
    const float* const* pre_ff_ln;
    const float* const* post_ff_ln;
    const float* const* q_proj;
    const float* const* k_proj;
    const float* const* v_proj;
    const float* const* o_proj;
    const float* const* q_norm;
    const float* const* k_norm;
    const float* const* gate_proj;
    const float* const* up_proj;
    const float* const* down_proj;
    const float* const* ple_gate;
    const float* const* ple_proj;
    const float* const* ple_post_norm;
    const float* final_norm;
    const float* ple_model_proj;
    const float* ple_norm;
    const float* embed_proj;
} eg2o_text;

static void add_inplace(float* a, const float* b, long n) {
#pragma omp parallel for schedule(static) if (n >= (1 << 15))
    for (long i = 0; i < n; i++) a[i] += b[i];
}

static void rope_rows(float* x, long rows, int heads, int hd, const float* cs, const float* sn) {
#pragma omp parallel for schedule(static) if (rows >= 256)
    for (long t = 0; t < rows; t++)
        for (int h = 0; h < heads; h++) rope_apply(x + (t * heads + h) * hd, hd, cs + t * hd, sn + t * hd);
}

int eg2o_text_forward_packed(const eg2o_text* m, const float* embeds, const int64_t* lens, int n_seq, float* out) {
    int h = m->hidden, p = m->ple_dim, nl = m->n_layers, nh = m->n_heads, ff = m->inter;
    long seq = 0;
    for (int s = 0; s < n_seq; s++) {
        if (lens[s] <= 0) return -1;
        seq += lens[s];
    }
    if (seq == 0) return 0;

    float* ple = (float*)malloc(sizeof(float) * seq * nl * p);
    eg2o_sgemm_nt((int)seq, nl * p, h, embeds, m->ple_model_proj, ple);
    float ple_scale = powf((float)h, -0.5f);
#pragma omp parallel for schedule(static)
    for (long i = 0; i < seq * nl * p; i++) ple[i] *= ple_scale;
    eg2o_rms_norm(ple, seq * nl, p, m->ple_norm, m->eps);

    float* positions = (float*)malloc(sizeof(float) * seq);
    {
        long r = 0;
        for (int s = 0; s < n_seq; s++)
            for (long i = 0; i < lens[s]; i++) positions[r++] = (float)i;
    }
    /* One cos/sin table per distinct (theta, head_dim), like the reference's rope_cache. */
    int maxhd = 0;
    for (int i = 0; i < nl; i++)
        if (m->head_dim[i] > maxhd) maxhd = m->head_dim[i];
    double* keys_theta = (double*)malloc(sizeof(double) * nl);
    int* keys_hd = (int*)malloc(sizeof(int) * nl);
    float** tab_c = (float**)calloc(nl, sizeof(float*));
    float** tab_s = (float**)calloc(nl, sizeof(float*));
    int n_keys = 0;
    int* layer_tab = (int*)malloc(sizeof(int) * nl);
    for (int i = 0; i < nl; i++) {
        int found = -1;
        for (int j = 0; j < n_keys; j++)
            if (keys_theta[j] == m->theta[i] && keys_hd[j] == m->head_dim[i]) found = j;
        if (found < 0) {
            int hd = m->head_dim[i];
            float* inv = (float*)malloc(sizeof(float) * hd / 2);
            rope_inv_freq(m->theta[i], hd, inv);
            tab_c[n_keys] = (float*)malloc(sizeof(float) * seq * hd);
            tab_s[n_keys] = (float*)malloc(sizeof(float) * seq * hd);
            rope_tables(positions, seq, inv, hd / 2, tab_c[n_keys], tab_s[n_keys]);
            free(inv);
            keys_theta[n_keys] = m->theta[i];
            keys_hd[n_keys] = hd;
            found = n_keys++;
        }
        layer_tab[i] = found;
    }

    float* hidden = (float*)malloc(sizeof(float) * seq * h);
    memcpy(hidden, embeds, sizeof(float) * seq * h);
    float* x = (float*)malloc(sizeof(float) * seq * h);
    float* q = (float*)malloc(sizeof(float) * seq * nh * maxhd);
    float* kk = (float*)malloc(sizeof(float) * seq * nh * maxhd);
    float* vv = (float*)malloc(sizeof(float) * seq * nh * maxhd);
    float* a = (float*)malloc(sizeof(float) * seq * nh * maxhd);
    float* o = (float*)malloc(sizeof(float) * seq * h);
    float* gate = (float*)malloc(sizeof(float) * seq * ff);
    float* up = (float*)malloc(sizeof(float) * seq * ff);
    float* g = (float*)malloc(sizeof(float) * seq * p);

    for (int i = 0; i < nl; i++) {
        int hd = m->head_dim[i], nkv = m->n_kv[i];
        const float* cs = tab_c[layer_tab[i]];
        const float* sn = tab_s[layer_tab[i]];
        /* attention sub-block */
        memcpy(x, hidden, sizeof(float) * seq * h);
        eg2o_rms_norm(x, seq, h, m->input_ln[i], m->eps);
        eg2o_sgemm_nt((int)seq, nh * hd, h, x, m->q_proj[i], q);
        eg2o_sgemm_nt((int)seq, nkv * hd, h, x, m->k_proj[i], kk);
        eg2o_sgemm_nt((int)seq, nkv * hd, h, x, m->v_proj[i], vv);
        eg2o_rms_norm(q, seq * nh, hd, m->q_norm[i], m->eps);
        eg2o_rms_norm(kk, seq * nkv, hd, m->k_norm[i], m->eps);
        eg2o_rms_norm(vv, seq * nkv, hd, NULL, m->eps);
        rope_rows(q, seq, nh, hd, cs, sn);
        rope_rows(kk, seq, nkv, hd, cs, sn);
        eg2o_attention_packed(q, kk, vv, lens, n_seq, nh, nkv, hd, m->sliding[i] ? m->window : -1, a);
        eg2o_sgemm_nt((int)seq, h, nh * hd, a, m->o_proj[i], o);
        eg2o_rms_norm(o, seq, h, m->post_attn_ln[i], m->eps);
        add_inplace(hidden, o, seq * h);
        /* feed-forward sub-block */
        memcpy(x, hidden, sizeof(float) * seq * h);
        eg2o_rms_norm(x, seq, h, m->pre_ff_ln[i], m->eps);
        eg2o_sgemm_nt((int)seq, ff, h, x, m->gate_proj[i], gate);
        eg2o_sgemm_nt((int)seq, ff, h, x, m->up_proj[i], up);
#pragma omp parallel for schedule(static)
        for (long j = 0; j < seq * ff; j++) gate[j] = gelu_tanh(gate[j]) * up[j];
        eg2o_sgemm_nt((int)seq, h, ff, gate, m->down_proj[i], o);
        eg2o_rms_norm(o, seq, h, m->post_ff_ln[i], m->eps);
        add_inplace(hidden, o, seq * h);
        /* per-layer-input sub-block */
        eg2o_sgemm_nt((int)seq, p, h, hidden, m->ple_gate[i], g);
#pragma omp parallel for schedule(static)
        for (long t = 0; t < seq; t++) {
            const float* pli = ple + (t * nl + i) * p;
            float* row = g + t * p;
            for (int c = 0; c < p; c++) row[c] = gelu_tanh(row[c]) * pli[c];
        }
        eg2o_sgemm_nt((int)seq, h, p, g, m->ple_proj[i], o);
        eg2o_rms_norm(o, seq, h, m->ple_post_norm[i], m->eps);
        add_inplace(hidden, o, seq * h);
        float ls = m->layer_scalar[i];
#pragma omp parallel for schedule(static)
        for (long j = 0; j < seq * h; j++) hidden[j] *= ls;
    }
    eg2o_rms_norm(hidden, seq, h, m->final_norm, m->eps);
    eg2o_sgemm_nt((int)seq, m->emb_dim, h, hidden, m->embed_proj, out);

    for (int j = 0; j < n_keys; j++) {
        free(tab_c[j]);
        free(tab_s[j]);
    }
    free(tab_c); free(tab_s); free(keys_theta); free(keys_hd); free(layer_tab); free(positions);
    free(ple); free(hidden); free(x); free(q); free(kk); free(vv); free(a); free(o); free(gate); free(up); free(g);
    return 0;
}

/* ------------------------------------------------------------------------------------------ */
/* Embedding gather, pooling, Matryoshka                                                       */
/* ------------------------------------------------------------------------------------------ */

/* src/text.rs:53-64: bf16 table row -> f32, times sqrt(h). */
int eg2o_embed_tokens(const uint16_t* table, long vocab, int h, const uint32_t* ids, long n, float* out) {
    float scale = sqrtf((float)h);
    for (long t = 0; t < n; t++) {
        if ((long)ids[t] >= vocab) return -1;
        const uint16_t* row = table + (long)ids[t] * h;
        for (int c = 0; c < h; c++) {
            uint32_t u = (uint32_t)row[c] << 16;
            float f;
            memcpy(&f, &u, 4);
            out[t * h + c] = f * scale;
        }
    }
    return 0;
}

/* src/ops.rs:462-467 */
void eg2o_l2_normalize(float* v, int n) {
    double ss = 0.0;
    for (int i = 0; i < n; i++) ss += (double)v[i] * (double)v[i];
    double norm = sqrt(ss);
    if (norm < 1e-12) norm = 1e-12;
    for (int i = 0; i < n; i++) v[i] = (float)((double)v[i] / norm);
}

/* Per sequence: mean_rows (f64) then l2_normalize (src/model.rs:530-535, src/ops.rs:451-467). */
void eg2o_pool(const float* hidden, const int64_t* lens, int n_seq, int dim, float* out) {
    long off = 0;
    double* acc = (double*)malloc(sizeof(double) * dim);
    for (int s = 0; s < n_seq; s++) {
        for (int c = 0; c < dim; c++) acc[c] = 0.0;
        for (long r = 0; r < lens[s]; r++)
            for (int c = 0; c < dim; c++) acc[c] += (double)hidden[(off + r) * dim + c];
        for (int c = 0; c < dim; c++) out[(long)s * dim + c] = (float)(acc[c] / (double)lens[s]);
        eg2o_l2_normalize(out + (long)s * dim, dim);
        off += lens[s];
    }
    free(acc);
}

/* ------------------------------------------------------------------------------------------ */
/* Vision tower (src/vision.rs:223-293)                                                        */
/* ------------------------------------------------------------------------------------------ */

typedef struct {
    int hidden, inter, n_layers, n_heads, n_kv, head_dim, patch_dim, pool_k, pos_size, text_hidden;
    float eps;
    double theta;
    const float* pos_table;   /* [2, pos_size, hidden] */
    const float* input_proj;  /* [hidden, patch_dim] */
    const float* embed_proj;  /* [text_hidden, hidden] */
    const float* const* q_proj;
    const float* const* k_proj;
    const float* const* v_proj;
    const float* const* o_proj;
    const float* const* q_norm;
    const float* const* k_norm;
    const float* const* gate_proj;
    const float* const* up_proj;
    const float* const* down_proj;
    const float* const* input_ln;
    const float* const* post_attn_ln;
    const float* const* pre_ff_ln;
    const float* const* post_ff_ln;
} eg2o_vision;

/* Pooled, sqrt(h)-scaled states before the embedder (src/vision.rs:140-163), then optionally
 * the embedder (scale-free RMSNorm + projection, src/vision.rs:167-170). out_pooled may be NULL. */
int eg2o_vision_encode(const eg2o_vision* m, const float* patches, const int32_t* pos_xy, int grid_h, int grid_w,
                       float* out_pooled, float* out_soft) {
    int h = m->hidden, hd = m->head_dim, nh = m->n_heads, nkv = m->n_kv, ff = m->inter, k = m->pool_k;
    long n = (long)grid_h * grid_w;
    if (n == 0 || grid_h % k || grid_w % k) return -1;
    for (long t = 0; t < n; t++)
        if (pos_xy[2 * t] < 0 || pos_xy[2 * t] >= m->pos_size || pos_xy[2 * t + 1] < 0 || pos_xy[2 * t + 1] >= m->pos_size)
            return -2;
    float* sp = (float*)malloc(sizeof(float) * n * m->patch_dim);
    for (long i = 0; i < n * m->patch_dim; i++) sp[i] = 2.0f * (patches[i] - 0.5f);
    float* hidden = (float*)malloc(sizeof(float) * n * h);
    eg2o_sgemm_nt((int)n, h, m->patch_dim, sp, m->input_proj, hidden);
    free(sp);
    for (long t = 0; t < n; t++) {
        const float* px = m->pos_table + (long)pos_xy[2 * t] * h;
        const float* py = m->pos_table + ((long)m->pos_size + pos_xy[2 * t + 1]) * h;
        for (int i = 0; i < h; i++) hidden[t * h + i] += px[i] + py[i];
    }
    /* Axial RoPE tables [n, hd] (src/vision.rs:114-136). */
    int hs = hd / 4;
    float* inv = (float*)malloc(sizeof(float) * hs);
    rope_inv_freq(m->theta, hd / 2, inv);
    float* cs = (float*)calloc(n * hd, sizeof(float));
    float* sn = (float*)calloc(n * hd, sizeof(float));
    for (long t = 0; t < n; t++)
        for (int axis = 0; axis < 2; axis++) {
            int pos = pos_xy[2 * t + axis];
            for (int i = 0; i < hs; i++) {
                float f = (float)pos * inv[i];
                float s = sinf(f), c = cosf(f);
                long base = t * hd + axis * (hd / 2);
                cs[base + i] = c;
                cs[base + hs + i] = c;
                sn[base + i] = s;
                sn[base + hs + i] = s;
            }
        }
    free(inv);
    float* x = (float*)malloc(sizeof(float) * n * h);
    float* q = (float*)malloc(sizeof(float) * n * nh * hd);
    float* kk = (float*)malloc(sizeof(float) * n * nkv * hd);
    float* vv = (float*)malloc(sizeof(float) * n * nkv * hd);
    float* a = (float*)malloc(sizeof(float) * n * nh * hd);
    float* o = (float*)malloc(sizeof(float) * n * h);
    float* gate = (float*)malloc(sizeof(float) * n * ff);
    float* up = (float*)malloc(sizeof(float) * n * ff);
    int64_t len1 = n;
    int part = hd / 2;
    for (int l = 0; l < m->n_layers; l++) {
        memcpy(x, hidden, sizeof(float) * n * h);
        eg2o_rms_norm(x, n, h, m->input_ln[l], m->eps);
        eg2o_sgemm_nt((int)n, nh * hd, h, x, m->q_proj[l], q);
        eg2o_sgemm_nt((int)n, nkv * hd, h, x, m->k_proj[l], kk);
        eg2o_sgemm_nt((int)n, nkv * hd, h, x, m->v_proj[l], vv);
        eg2o_rms_norm(q, n * nh, hd, m->q_norm[l], m->eps);
        eg2o_rms_norm(kk, n * nkv, hd, m->k_norm[l], m->eps);
        eg2o_rms_norm(vv, n * nkv, hd, NULL, m->eps);
        /* rope_2d (src/vision.rs:278-293) */
#pragma omp parallel for schedule(static)
        for (long t = 0; t < n; t++) {
            for (int hh = 0; hh < nh; hh++)
                for (int axis = 0; axis < 2; axis++)
                    rope_apply(q + (t * nh + hh) * hd + axis * part, part, cs + t * hd + axis * part, sn + t * hd + axis * part);
            for (int hh = 0; hh < nkv; hh++)
                for (int axis = 0; axis < 2; axis++)
                    rope_apply(kk + (t * nkv + hh) * hd + axis * part, part, cs + t * hd + axis * part, sn + t * hd + axis * part);
        }
        eg2o_attention_packed(q, kk, vv, &len1, 1, nh, nkv, hd, -1, a);
        eg2o_sgemm_nt((int)n, h, nh * hd, a, m->o_proj[l], o);
        eg2o_rms_norm(o, n, h, m->post_attn_ln[l], m->eps);
        add_inplace(hidden, o, n * h);
        memcpy(x, hidden, sizeof(float) * n * h);
        eg2o_rms_norm(x, n, h, m->pre_ff_ln[l], m->eps);
        eg2o_sgemm_nt((int)n, ff, h, x, m->gate_proj[l], gate);
        eg2o_sgemm_nt((int)n, ff, h, x, m->up_proj[l], up);
#pragma omp parallel for schedule(static)
        for (long j = 0; j < n * ff; j++) gate[j] = gelu_tanh(gate[j]) * up[j];
        eg2o_sgemm_nt((int)n, h, ff, gate, m->down_proj[l], o);
        eg2o_rms_norm(o, n, h, m->post_ff_ln[l], m->eps);
        add_inplace(hidden, o, n * h);
    }
    /* pool_and_embed (src/vision.rs:140-170) */
    int oh = grid_h / k, ow = grid_w / k;
    float root = sqrtf((float)h);
    float* pooled = (float*)malloc(sizeof(float) * (long)oh * ow * h);
    for (int ob = 0; ob < oh * ow; ob++) {
        int oy = ob / ow, ox = ob % ow;
        float* acc = pooled + (long)ob * h;
        for (int c = 0; c < h; c++) acc[c] = 0.f;
        for (int dy = 0; dy < k; dy++)
            for (int dx = 0; dx < k; dx++) {
                long t = (long)(oy * k + dy) * grid_w + ox * k + dx;
                for (int c = 0; c < h; c++) acc[c] += hidden[t * h + c];
            }
        float denom = (float)(k * k);
        for (int c = 0; c < h; c++) acc[c] = (acc[c] / denom) * root;
    }
    if (out_pooled) memcpy(out_pooled, pooled, sizeof(float) * (long)oh * ow * h);
    if (out_soft) {
        eg2o_rms_norm(pooled, (long)oh * ow, h, NULL, m->eps);
        eg2o_sgemm_nt(oh * ow, m->text_hidden, h, pooled, m->embed_proj, out_soft);
    }
    free(pooled); free(cs); free(sn); free(hidden); free(x); free(q); free(kk); free(vv); free(a); free(o); free(gate);
    free(up);
    return 0;
}

int eg2o_num_threads(void) { return omp_get_max_threads(); }
void eg2o_set_threads(int n) {
    if (n > 0) omp_set_num_threads(n);
}
