/*
 * gqa_oracle.c -- CPU restatement of the reference's GQA attention core.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA kernels
 * are compared against; nothing in the product path links or calls it.  Only
 * tests/, __graft_entry__.smoke() and the cpu_baseline / reference legs of
 * bench.py may load it.
 *
 * It restates, stage by stage, the bf16-staged arithmetic of
 * llama3_attention_golden_model.py (reference repository):
 *   to_bf16                 :44-47   -> orc_f32_to_bf16 (round-to-nearest-even)
 *   build_rope_cache        :124-130 -> orc_rope_table
 *   rotate_half/apply_rope  :133-139, used :162-164 -> orc_rope_apply
 *   scores = QK^T * scale   :175-176 -> orc_scores
 *   causal mask             :180-181 -> orc_mask_golden
 *   softmax                 :185     -> orc_softmax
 *   PV                      :189     -> orc_pv
 * and the HLS mask kernel attention_mask_module/src/attention_mask.cpp:3-58
 * (raw 16-bit word pass-through, mask word above the diagonal) ->
 * orc_attention_mask_words.
 *
 * Arithmetic conventions (each one checked against the reference's committed
 * hex golden vectors by tests/test_oracle_golden.py):
 *  - bf16 <-> fp32 conversions are exact widening / RNE narrowing, NaN -> 0x7FC0.
 *  - RoPE angles are fp32 products pos*inv_freq with inv_freq = 1/fl32(theta^(2i/d));
 *    cos/sin are evaluated in double precision on that fp32 angle and rounded
 *    to fp32, then to bf16 (matches torch's fp32 tables bit-exactly for
 *    positions < 8192).
 *  - x*cos and rotate_half(x)*sin are exact in fp32 (bf16*bf16); their sum is
 *    one fp32 rounding, then RNE to bf16.
 *  - dot products accumulate in fp32 in key/dim order (the golden's sgemm order
 *    is library-defined; the hex goldens pin the effect at the bf16 boundary).
 *  - the score is fl32(fl32(dot) * fl32(1/sqrt(d))), then bf16.
 *  - masked positions add -inf; unmasked add +0.0 (so -0.0 becomes +0.0).
 *  - softmax: fp32 max, exp in double rounded to fp32, fp32 sum, fp32 divide.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <pthread.h>
#include <stdlib.h>
#include <unistd.h>

/* ---- minimal static-partition parallel-for over [0, n) on pthreads ---- */
typedef void (*orc_body_fn)(long begin, long end, void* ctx);
typedef struct { orc_body_fn fn; void* ctx; long begin, end; } orc_job;

static int g_threads = 0;

void orc_set_num_threads(int n) { g_threads = n; }

int orc_num_threads(void) {
    if (g_threads > 0) return g_threads;
    const char* e = getenv("ORACLE_THREADS");
    if (e && atoi(e) > 0) return atoi(e);
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

static void* orc_worker(void* p) {
    orc_job* j = (orc_job*)p;
    j->fn(j->begin, j->end, j->ctx);
    return NULL;
}

static void orc_parallel_for(long n, orc_body_fn fn, void* ctx) {
    int nt = orc_num_threads();
    if (nt > 256) nt = 256;
    if (nt <= 1 || n < 2) { fn(0, n, ctx); return; }
    if (nt > n) nt = (int)n;
    pthread_t th[256];
    orc_job jobs[256];
    long chunk = (n + nt - 1) / nt;
    int started = 0;
    for (int t = 0; t < nt; ++t) {
        long b = t * chunk, e = b + chunk < n ? b + chunk : n;
        if (b >= e) break;
        jobs[t].fn = fn; jobs[t].ctx = ctx; jobs[t].begin = b; jobs[t].end = e;
        if (t == 0) continue;
        if (pthread_create(&th[t], NULL, orc_worker, &jobs[t]) != 0) { fn(b, e, ctx); jobs[t].fn = NULL; }
        started = t;
    }
    fn(jobs[0].begin, jobs[0].end, ctx);
    for (int t = 1; t <= started; ++t)
        if (jobs[t].fn) pthread_join(th[t], NULL);
}

static inline float bf2f(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint16_t f2bf(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return 0x7FC0;
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

uint16_t orc_f32_to_bf16(float f) { return f2bf(f); }
float orc_bf16_to_f32(uint16_t h) { return bf2f(h); }

void orc_f32_to_bf16_array(const float* x, uint16_t* y, long n) {
    for (long i = 0; i < n; ++i) y[i] = f2bf(x[i]);
}

void orc_bf16_to_f32_array(const uint16_t* x, float* y, long n) {
    for (long i = 0; i < n; ++i) y[i] = bf2f(x[i]);
}

/* inv_freq[i] = 1 / fl32(theta ** (2i/d)), all in fp32 as the golden does. */
void orc_inv_freq(int dim, double theta, float* inv_freq) {
    for (int i = 0; i < dim / 2; ++i) {
        float e = (float)(2 * i) / (float)dim;
        float p = (float)pow(theta, (double)e);
        inv_freq[i] = 1.0f / p;
    }
}

/* cos/sin tables [S][dim] (emb = cat(freqs, freqs)) for positions pos0..pos0+S-1. */
void orc_rope_table(int S, int pos0, int dim, double theta, uint16_t* cos_tab, uint16_t* sin_tab) {
    float inv[512];
    orc_inv_freq(dim, theta, inv);
    int half = dim / 2;
    for (int s = 0; s < S; ++s) {
        float pos = (float)(pos0 + s);
        for (int i = 0; i < half; ++i) {
            float ang = pos * inv[i];
            uint16_t c = f2bf((float)cos((double)ang));
            uint16_t sn = f2bf((float)sin((double)ang));
            cos_tab[(long)s * dim + i] = c;
            cos_tab[(long)s * dim + i + half] = c;
            sin_tab[(long)s * dim + i] = sn;
            sin_tab[(long)s * dim + i + half] = sn;
        }
    }
}

/* y[h][s][:] = bf16(x*cos + rotate_half(x)*sin); x,y [H][S][D], tables [S][D]. */
void orc_rope_apply(const uint16_t* x, uint16_t* y, const uint16_t* cos_tab, const uint16_t* sin_tab,
                    int H, int S, int D) {
    int half = D / 2;
    for (int h = 0; h < H; ++h)
        for (int s = 0; s < S; ++s) {
            const uint16_t* xr = x + ((long)h * S + s) * D;
            uint16_t* yr = y + ((long)h * S + s) * D;
            const uint16_t* cr = cos_tab + (long)s * D;
            const uint16_t* sr = sin_tab + (long)s * D;
            for (int d = 0; d < D; ++d) {
                float xv = bf2f(xr[d]);
                float rv = d < half ? -bf2f(xr[d + half]) : bf2f(xr[d - half]);
                float a = xv * bf2f(cr[d]);
                float b = rv * bf2f(sr[d]);
                yr[d] = f2bf(a + b);
            }
        }
}

/* scores[hq][i][j] = bf16(fl32(q[hq][i].k[hq/G][j]) * fl32(scale)); [Hq][S][S]. */
typedef struct { const uint16_t *q, *k; uint16_t* out; int Hq, Hkv, S, D; float scale; } scores_ctx;

static void scores_body(long b, long e, void* p) {
    scores_ctx* c = (scores_ctx*)p;
    int G = c->Hq / c->Hkv, S = c->S, D = c->D;
    float qf[1024];
    for (long r = b; r < e; ++r) {
        int h = (int)(r / S), i = (int)(r % S);
        const uint16_t* qr = c->q + ((long)h * S + i) * D;
        for (int d = 0; d < D; ++d) qf[d] = bf2f(qr[d]);
        const uint16_t* kb = c->k + (long)(h / G) * S * D;
        uint16_t* orow = c->out + ((long)h * S + i) * S;
        for (int j = 0; j < S; ++j) {
            const uint16_t* kr = kb + (long)j * D;
            float acc = 0.0f;
            for (int d = 0; d < D; ++d) acc += qf[d] * bf2f(kr[d]);
            orow[j] = f2bf(acc * c->scale);
        }
    }
}

void orc_scores(const uint16_t* q, const uint16_t* k, uint16_t* out, int Hq, int Hkv, int S, int D,
                float scale) {
    scores_ctx c = {q, k, out, Hq, Hkv, S, D, scale};
    orc_parallel_for((long)Hq * S, scores_body, &c);
}

/* golden mask: bf16(score + (j > i ? -inf : +0.0)). in/out [H][S][S]. */
void orc_mask_golden(const uint16_t* in, uint16_t* out, int H, int S, int causal) {
    for (int h = 0; h < H; ++h)
        for (int i = 0; i < S; ++i)
            for (int j = 0; j < S; ++j) {
                long idx = ((long)h * S + i) * S + j;
                float m = (causal && j > i) ? -INFINITY : 0.0f;
                out[idx] = f2bf(bf2f(in[idx]) + m);
            }
}

/* HLS mask kernel: raw 16-bit word pass-through, mask_value above the diagonal.
 * Returns 0 on success, -1 on invalid sizes (the HLS kernel returns silently). */
int orc_attention_mask_words(const uint16_t* raw, uint16_t* masked, int q_heads, int seq_len, int causal,
                             uint16_t mask_value) {
    if (q_heads <= 0 || seq_len <= 0) return -1;
    long idx = 0;
    for (int h = 0; h < q_heads; ++h)
        for (int qt = 0; qt < seq_len; ++qt)
            for (int kt = 0; kt < seq_len; ++kt, ++idx)
                masked[idx] = (causal && kt > qt) ? mask_value : raw[idx];
    return 0;
}

/* softmax over the last axis: in [rows][cols] bf16 -> out bf16. */
typedef struct { const uint16_t* in; uint16_t* out; int cols; } softmax_ctx;

static void softmax_body(long b, long e, void* p) {
    softmax_ctx* c = (softmax_ctx*)p;
    int cols = c->cols;
    float* ex = (float*)malloc(sizeof(float) * (size_t)cols);
    for (long r = b; r < e; ++r) {
        const uint16_t* x = c->in + r * cols;
        uint16_t* y = c->out + r * cols;
        float mx = -INFINITY;
        for (int j = 0; j < cols; ++j) {
            float v = bf2f(x[j]);
            if (v > mx) mx = v;
        }
        float sum = 0.0f;
        for (int j = 0; j < cols; ++j) {
            float t = bf2f(x[j]) - mx;
            ex[j] = (float)exp((double)t);
            sum += ex[j];
        }
        for (int j = 0; j < cols; ++j) y[j] = f2bf(ex[j] / sum);
    }
    free(ex);
}

void orc_softmax(const uint16_t* in, uint16_t* out, long rows, int cols) {
    softmax_ctx c = {in, out, cols};
    orc_parallel_for(rows, softmax_body, &c);
}

/* out[hq][i][:] = bf16(sum_j fl32 p[hq][i][j] * v[hq/G][j][:]) accumulated in j order. */
typedef struct { const uint16_t *p, *v; uint16_t* out; int Hq, Hkv, S, D; } pv_ctx;

static void pv_body(long b, long e, void* p) {
    pv_ctx* c = (pv_ctx*)p;
    int G = c->Hq / c->Hkv, S = c->S, D = c->D;
    float acc[1024];
    for (long r = b; r < e; ++r) {
        int h = (int)(r / S), i = (int)(r % S);
        for (int d = 0; d < D; ++d) acc[d] = 0.0f;
        const uint16_t* pr = c->p + ((long)h * S + i) * S;
        const uint16_t* vb = c->v + (long)(h / G) * S * D;
        for (int j = 0; j < S; ++j) {
            float pj = bf2f(pr[j]);
            const uint16_t* vr = vb + (long)j * D;
            for (int d = 0; d < D; ++d) acc[d] += pj * bf2f(vr[d]);
        }
        uint16_t* orow = c->out + ((long)h * S + i) * D;
        for (int d = 0; d < D; ++d) orow[d] = f2bf(acc[d]);
    }
}

void orc_pv(const uint16_t* p, const uint16_t* v, uint16_t* out, int Hq, int Hkv, int S, int D) {
    pv_ctx c = {p, v, out, Hq, Hkv, S, D};
    orc_parallel_for((long)Hq * S, pv_body, &c);
}

/*
 * Exact attention for selected query rows, double-precision accumulation.
 * q [Hq][Sq][D] bf16 (already rotated), k/v [Hkv][Sk][D] bf16 (k rotated).
 * rows: n_rows (head, position) pairs; out [n_rows][D] fp32.
 * causal: keys j <= position are attended.  n_keys (if non-NULL) caps the key
 * range per row (decode: a cache of length L attends keys [0, L)).
 * Used to check long-sequence and decode outputs on sampled rows.
 */
typedef struct {
    const uint16_t *q, *k, *v;
    int Hq, Hkv, Sq, Sk, D;
    float scale;
    int causal;
    const int *row_head, *row_pos, *n_keys;
    float* out;
} rows_ctx;

static void rows_body(long b, long e, void* p) {
    rows_ctx* c = (rows_ctx*)p;
    int G = c->Hq / c->Hkv, D = c->D;
    double* sc = (double*)malloc(sizeof(double) * (size_t)(c->Sk > 0 ? c->Sk : 1));
    double o[1024];
    for (long r = b; r < e; ++r) {
        int h = c->row_head[r], i = c->row_pos[r];
        const uint16_t* qr = c->q + ((long)h * c->Sq + i) * D;
        const uint16_t* kb = c->k + (long)(h / G) * c->Sk * D;
        const uint16_t* vb = c->v + (long)(h / G) * c->Sk * D;
        int nk = c->Sk;
        if (c->causal && i + 1 < nk) nk = i + 1;
        if (c->n_keys && c->n_keys[r] < nk) nk = c->n_keys[r];
        double mx = -INFINITY;
        for (int j = 0; j < nk; ++j) {
            double acc = 0.0;
            const uint16_t* kr = kb + (long)j * D;
            for (int d = 0; d < D; ++d) acc += (double)bf2f(qr[d]) * (double)bf2f(kr[d]);
            sc[j] = acc * (double)c->scale;
            if (sc[j] > mx) mx = sc[j];
        }
        for (int d = 0; d < D; ++d) o[d] = 0.0;
        double l = 0.0;
        for (int j = 0; j < nk; ++j) {
            double pj = exp(sc[j] - mx);
            l += pj;
            const uint16_t* vr = vb + (long)j * D;
            for (int d = 0; d < D; ++d) o[d] += pj * (double)bf2f(vr[d]);
        }
        for (int d = 0; d < D; ++d) c->out[r * D + d] = (float)(l > 0 ? o[d] / l : 0.0);
    }
    free(sc);
}

void orc_attention_rows(const uint16_t* q, const uint16_t* k, const uint16_t* v, int Hq, int Hkv, int Sq,
                        int Sk, int D, float scale, int causal, const int* row_head, const int* row_pos,
                        const int* n_keys, int n_rows, float* out) {
    rows_ctx c = {q, k, v, Hq, Hkv, Sq, Sk, D, scale, causal, row_head, row_pos, n_keys, out};
    orc_parallel_for(n_rows, rows_body, &c);
}
