/*
 * TEST INFRASTRUCTURE - the CPU oracle for the decode-step kernel set. Not product code: only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs load it,
 * and only as the checker or as the timed CPU baseline, never on the product path.
 *
 * Each function restates one of the reference's own CPU checks, in plain C, with the arithmetic
 * those checks use (float products, float or double sums in the same order). It is compiled with
 * -ffp-contract=off so that `sum += a * b` stays a rounded multiply and a rounded add, as in the
 * reference's C++ loops. Reference citations are relative to the muyo-llm project root.
 *
 * Pinning: tests/test_oracle.py checks every function here against the reference's known answers
 * (the integer patterns of src/MatVec.cpp, src/ElementwiseAdd.cpp, src/GetRows.cpp,
 * src/Argmax.cpp, which are exact) and against golden vectors produced by running the unmodified
 * tools/reference_qwen2.py (tests/golden/make_golden.py).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* Row-parallel helper: rows are split into contiguous ranges, one per thread. Each row is still
 * summed sequentially by one thread, so the thread count never changes a result. */
static int g_threads = 1;
static pthread_mutex_t g_h2f_lock = PTHREAD_MUTEX_INITIALIZER;

typedef void (*row_fn)(void* ctx, int r0, int r1);
typedef struct {
    row_fn fn;
    void* ctx;
    int r0, r1;
} row_task;

static void* row_task_main(void* p)
{
    row_task* t = (row_task*)p;
    t->fn(t->ctx, t->r0, t->r1);
    return NULL;
}

static void parallel_rows(row_fn fn, void* ctx, int rows)
{
    int nt = g_threads;
    if (nt > 64)
        nt = 64;
    if (nt <= 1 || rows < 64) {
        fn(ctx, 0, rows);
        return;
    }
    pthread_t tid[64];
    row_task task[64];
    int created[64] = {0};
    const int chunk = ((rows + nt - 1) / nt + 3) / 4 * 4;
    int ntasks = 0;
    for (int i = 0; i < nt; ++i) {
        const int r0 = i * chunk, r1 = (i + 1) * chunk < rows ? (i + 1) * chunk : rows;
        if (r0 >= r1)
            break;
        task[i] = (row_task){fn, ctx, r0, r1};
        ntasks = i + 1;
        if (i > 0)
            created[i] = pthread_create(&tid[i], NULL, row_task_main, &task[i]) == 0;
    }
    fn(ctx, task[0].r0, task[0].r1);
    for (int i = 1; i < ntasks; ++i) {
        if (created[i])
            pthread_join(tid[i], NULL);
        else
            row_task_main(&task[i]);
    }
}

/* ---- F16 conversion -------------------------------------------------------------------------- */

static float g_h2f[65536];
static int g_h2f_ready = 0;

/* IEEE binary16 -> binary32, exact (normals, subnormals, inf, nan). */
static float h2f_slow(uint16_t h)
{
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1fu;
    const uint32_t man = h & 0x3ffu;
    float v;
    if (exp == 0)
        v = ldexpf((float)man, -24);
    else if (exp == 31)
        v = man ? NAN : INFINITY;
    else
        v = ldexpf((float)(man | 0x400u), (int)exp - 25);
    uint32_t bits;
    memcpy(&bits, &v, 4);
    bits |= sign;
    memcpy(&v, &bits, 4);
    return v;
}

static void h2f_init(void)
{
    if (__atomic_load_n(&g_h2f_ready, __ATOMIC_ACQUIRE))
        return;
    pthread_mutex_lock(&g_h2f_lock);
    if (!g_h2f_ready) {
        for (uint32_t i = 0; i < 65536u; ++i)
            g_h2f[i] = h2f_slow((uint16_t)i);
        __atomic_store_n(&g_h2f_ready, 1, __ATOMIC_RELEASE);
    }
    pthread_mutex_unlock(&g_h2f_lock);
}

static inline float h2f(uint16_t h) { return g_h2f[h]; }

/* binary32 -> binary16, round to nearest even (what the F16 KV cache stores). */
uint16_t oracle_f2h(float f)
{
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) /* inf / nan */
        return sign | (ax > 0x7f800000u ? 0x7e00u : 0x7c00u);
    if (ax >= 0x477ff000u) /* rounds to >= 65520 -> inf */
        return sign | 0x7c00u;
    if (ax < 0x38800000u) { /* subnormal half (or zero) */
        /* value = ax as float; half subnormal unit is 2^-24 */
        float a;
        memcpy(&a, &ax, 4);
        const float scaled = a * 16777216.0f; /* exact: multiply by 2^24 */
        const float r = nearbyintf(scaled);  /* round half to even (default rounding mode) */
        return sign | (uint16_t)r;
    }
    /* normal: rebias exponent, round mantissa from 23 to 10 bits, ties to even */
    uint32_t m = ax - 0x38000000u; /* exponent rebias (127 - 15) << 23 */
    const uint32_t lsb = (m >> 13) & 1u;
    m += 0x0fffu + lsb;
    return sign | (uint16_t)(m >> 13);
}

float oracle_h2f(uint16_t h)
{
    h2f_init();
    return h2f(h);
}

void oracle_f2h_array(const float* x, uint16_t* y, int64_t n)
{
    for (int64_t i = 0; i < n; ++i)
        y[i] = oracle_f2h(x[i]);
}

/* ---- per-op checks ---------------------------------------------------------------------------- */

/* One GEMV row: the reference's HostMatVec (src/MatVec.cpp:52-60), a sequential float sum of
 * float(A16[row, k]) * b[k]. */
static inline float row_dot_f16(const uint16_t* a, const float* x, int cols)
{
    float sum = 0.0f;
    for (int k = 0; k < cols; ++k)
        sum += h2f(a[k]) * x[k];
    return sum;
}

/* Four rows at once: four independent sequential sums, each identical to row_dot_f16. */
static inline void row_dot4_f16(const uint16_t* a, size_t lda, const float* x, int cols, float out[4])
{
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    const uint16_t* a1 = a + lda;
    const uint16_t* a2 = a + 2 * lda;
    const uint16_t* a3 = a + 3 * lda;
    for (int k = 0; k < cols; ++k) {
        const float xk = x[k];
        s0 += h2f(a[k]) * xk;
        s1 += h2f(a1[k]) * xk;
        s2 += h2f(a2[k]) * xk;
        s3 += h2f(a3[k]) * xk;
    }
    out[0] = s0;
    out[1] = s1;
    out[2] = s2;
    out[3] = s3;
}

/* y[r] = sum_k A[r,k] x[k] (+ bias0[r]) (+ bias1[r]): src/MatVec.cpp:52-60 for the sum;
 * the BIAS0/BIAS1 fusion adds after the row sum (shaders/llama/mul_mat_vec_base.glsl:110-125,
 * src/LlamaContracts.h:109-118). Rows run in parallel; each row's sum is sequential. */
typedef struct {
    const uint16_t* a;
    int64_t lda;
    const float* x;
    float* y;
    int rows, cols;
    const float *bias0, *bias1;
} mat_vec_ctx;

static void mat_vec_rows(void* p, int begin, int end)
{
    const mat_vec_ctx* c = (const mat_vec_ctx*)p;
    const uint16_t* a = c->a;
    const int64_t lda = c->lda;
    const float* x = c->x;
    float* y = c->y;
    const int rows = end, cols = c->cols;
    const float *bias0 = c->bias0, *bias1 = c->bias1;
    for (int r0 = begin; r0 < rows; r0 += 4) {
        float s[4];
        if (r0 + 4 <= rows) {
            row_dot4_f16(a + (size_t)r0 * lda, (size_t)lda, x, cols, s);
        } else {
            for (int i = 0; i < rows - r0; ++i)
                s[i] = row_dot_f16(a + (size_t)(r0 + i) * lda, x, cols);
        }
        for (int i = 0; i < 4 && r0 + i < rows; ++i) {
            float v = s[i];
            if (bias0)
                v += bias0[r0 + i];
            if (bias1)
                v += bias1[r0 + i];
            y[r0 + i] = v;
        }
    }
}

void oracle_mat_vec_f16(const uint16_t* a, int64_t lda, const float* x, float* y, int rows, int cols,
                        const float* bias0, const float* bias1)
{
    h2f_init();
    mat_vec_ctx c = {a, lda, x, y, rows, cols, bias0, bias1};
    parallel_rows(mat_vec_rows, &c, rows);
}

/* Batched F32 GEMV with ggml's broadcast mapping (shaders/llama/mul_mat_vec_base.glsl:49-64):
 * batch b reads A batch (b / ne12 / broadcast3) * ne02 + (b % ne12) / broadcast2. Row sums as
 * src/TransformerLayer.cpp:209-223. */
void oracle_mat_vec_f32(const float* a, const float* b, float* d, int ncols, int rows, int batches,
                        int stride_a, int batch_stride_a, int batch_stride_b,
                        int batch_stride_d, int ne02, int ne12, int broadcast2, int broadcast3,
                        const float* bias0)
{
    for (int batch = 0; batch < batches; ++batch) {
        const int i13 = batch / ne12, i12 = batch % ne12;
        const int batch_a = (i13 / broadcast3) * ne02 + i12 / broadcast2;
        const float* A = a + (size_t)batch_a * batch_stride_a;
        const float* B = b + (size_t)batch * batch_stride_b;
        float* D = d + (size_t)batch * batch_stride_d;
        for (int r = 0; r < rows; ++r) {
            float sum = 0.0f;
            for (int k = 0; k < ncols; ++k)
                sum += A[(size_t)r * stride_a + k] * B[k];
            if (bias0)
                sum += bias0[(size_t)batch * batch_stride_d + r];
            D[r] = sum;
        }
    }
}

/* src/RmsNorm.cpp:194-205: double sum of squares, scale = float(1 / sqrt(ss / n + eps)),
 * y = x * scale * w (weight broadcast by column). */
void oracle_rms_norm(const float* x, const float* w, float* y, int rows, int cols, float eps)
{
    for (int r = 0; r < rows; ++r) {
        const float* xr = x + (size_t)r * cols;
        double ss = 0.0;
        for (int c = 0; c < cols; ++c)
            ss += (double)xr[c] * xr[c];
        const float scale = (float)(1.0 / sqrt(ss / cols + eps));
        for (int c = 0; c < cols; ++c)
            y[(size_t)r * cols + c] = xr[c] * scale * w[c];
    }
}

/* src/ElementwiseAdd.cpp:208. */
void oracle_add(const float* a, const float* b, float* d, int64_t n)
{
    for (int64_t i = 0; i < n; ++i)
        d[i] = a[i] + b[i];
}

/* src/Swiglu.cpp:56,187: silu(g) * u with silu(v) = v / (1 + exp(-v)). */
void oracle_swiglu(const float* g, const float* u, float* d, int64_t n)
{
    for (int64_t i = 0; i < n; ++i)
        d[i] = g[i] / (1.0f + expf(-g[i])) * u[i];
}

/* src/Rope.cpp:191-203 (and src/KvCache.cpp:78-91): NeoX pairs (j, j + n_dims/2), theta =
 * pos * theta_scale^j in float, theta_scale = base^(-2/n_dims) computed by the caller in float
 * (src/FullModel.cpp:201). Channels >= n_dims are copied. */
void oracle_rope_neox(const float* x, float* y, int rows, int ne00, int n_dims, int in_stride,
                      int out_stride, int pos, float theta_scale)
{
    const int half = n_dims / 2;
    for (int r = 0; r < rows; ++r) {
        const float* xr = x + (size_t)r * in_stride;
        float* yr = y + (size_t)r * out_stride;
        for (int j = 0; j < half; ++j) {
            const float theta = (float)pos * powf(theta_scale, (float)j);
            const float c = cosf(theta), s = sinf(theta);
            const float x0 = xr[j], x1 = xr[j + half];
            yr[j] = x0 * c - x1 * s;
            yr[j + half] = x0 * s + x1 * c;
        }
        for (int j = n_dims; j < ne00; ++j)
            yr[j] = xr[j];
    }
}

/* src/SoftMax.cpp:164-182: v = x * scale, max, double sum of float exp(v - max),
 * p = float(exp(v - max) / sum). */
void oracle_soft_max(const float* x, float* y, int rows, int cols, float scale)
{
    float* v = (float*)malloc(sizeof(float) * (size_t)cols);
    for (int r = 0; r < rows; ++r) {
        const float* xr = x + (size_t)r * cols;
        float m = -1e30f;
        for (int c = 0; c < cols; ++c) {
            v[c] = xr[c] * scale;
            m = v[c] > m ? v[c] : m;
        }
        double sum = 0.0;
        for (int c = 0; c < cols; ++c)
            sum += expf(v[c] - m);
        for (int c = 0; c < cols; ++c)
            y[(size_t)r * cols + c] = (float)(expf(v[c] - m) / sum);
    }
    free(v);
}

/* The greedy pick of src/Sampler.cpp:32-43: the first index of the maximum (strict >). */
int oracle_argmax(const float* x, int64_t n)
{
    int64_t best = 0;
    for (int64_t i = 1; i < n; ++i)
        if (x[i] > x[best])
            best = i;
    return (int)best;
}

/* src/GetRows.cpp:181, src/Embedding.cpp:70-77: out = float(table[token, :]). */
void oracle_get_rows_f16(const uint16_t* table, int dim, int token, float* out)
{
    h2f_init();
    for (int c = 0; c < dim; ++c)
        out[c] = h2f(table[(size_t)token * dim + c]);
}

/* src/Attention.cpp:254-285 for one query head over n keys: float dot products scaled,
 * max-subtracted float exp, double normaliser, float weighted sum over V. Keys and values are
 * row-major [n][hd]; `head` rows of q are served by kv head head / gqa (tools/reference_qwen2.py:133).
 */
void oracle_attention(const float* q, const float* keys, const float* values, float* out, int heads,
                      int kv_heads, int n, int hd, int kv_stride, float scale)
{
    const int gqa = heads / kv_heads;
    float* s = (float*)malloc(sizeof(float) * (size_t)n);
    for (int h = 0; h < heads; ++h) {
        const float* K = keys + (size_t)(h / gqa) * kv_stride;
        const float* V = values + (size_t)(h / gqa) * kv_stride;
        const float* qh = q + (size_t)h * hd;
        float m = -1e30f;
        for (int j = 0; j < n; ++j) {
            float dot = 0.0f;
            for (int d = 0; d < hd; ++d)
                dot += K[(size_t)j * hd + d] * qh[d];
            s[j] = dot * scale;
            m = s[j] > m ? s[j] : m;
        }
        double sum = 0.0;
        for (int j = 0; j < n; ++j) {
            s[j] = expf(s[j] - m);
            sum += s[j];
        }
        for (int j = 0; j < n; ++j)
            s[j] = (float)(s[j] / sum);
        for (int d = 0; d < hd; ++d) {
            float acc = 0.0f;
            for (int j = 0; j < n; ++j)
                acc += s[j] * V[(size_t)j * hd + d];
            out[(size_t)h * hd + d] = acc;
        }
    }
    free(s);
}

/* ---- Qwen2 decode step ----------------------------------------------------------------------- */

/* The whole-model forward of tools/reference_qwen2.py:107-168, restated in float (the arithmetic
 * of the reference's C++ engine, src/FullModel.cpp), one token at a time:
 *   x  = rms_norm(h)            x / sqrt(mean(x^2) + eps) * w            (reference_qwen2.py:81-82)
 *   q,k,v = W x + b; q,k = rope_neox(., pos)                             (:112-124, :84-93)
 *   append k, v to the cache (F32, or rounded to F16 when kv_f16)        (:126-130)
 *   attention per query head over kv head h / gqa, scale 1/sqrt(hd)      (:131-137)
 *   h += W_o attn; h += W_down (silu(W_gate x2) * W_up x2)              (:138-157)
 *   logits = W_out rms_norm(h)                                           (:160-163)
 * The rotation follows reference_qwen2.py:88-92 in double (theta = pos * base^(-2j/hd)), rounded
 * to float once. */
typedef struct OracleQwen2Layer {
    const float* attn_norm;
    const uint16_t* wq;
    const float* bq;
    const uint16_t* wk;
    const float* bk;
    const uint16_t* wv;
    const float* bv;
    const uint16_t* wo;
    const float* ffn_norm;
    const uint16_t* wgate;
    const uint16_t* wup;
    const uint16_t* wdown;
} OracleQwen2Layer;

typedef struct OracleQwen2 {
    int layers, hidden, ffn, heads, kv_heads, vocab, max_seq;
    float eps, rope_base;
    const uint16_t* token_embd;
    const uint16_t* output;
    const float* output_norm;
    const OracleQwen2Layer* layer;
} OracleQwen2;

static void qwen2_rms_norm(const float* x, const float* w, float* y, int n, float eps)
{
    double ss = 0.0;
    for (int i = 0; i < n; ++i)
        ss += (double)x[i] * x[i];
    const float mean = (float)(ss / n);
    const float s = sqrtf(mean + eps);
    for (int i = 0; i < n; ++i)
        y[i] = (x[i] / s) * w[i];
}

static void qwen2_rope(float* x, int heads, int hd, int pos, float base)
{
    const int half = hd / 2;
    for (int j = 0; j < half; ++j) {
        const double theta = (double)pos * pow((double)base, -2.0 * j / hd);
        const double c = cos(theta), s = sin(theta);
        for (int h = 0; h < heads; ++h) {
            float* xr = x + (size_t)h * hd;
            const double x0 = xr[j], x1 = xr[j + half];
            const double p0 = x0 * c, p1 = x1 * s, p2 = x0 * s, p3 = x1 * c;
            xr[j] = (float)(p0 - p1);
            xr[j + half] = (float)(p2 + p3);
        }
    }
}

/* One decoder layer at position pos: h is updated in place. The caches are
 * [kv_heads][max_seq][hd], F32 (kv_f16 = 0) or F16 bits (kv_f16 = 1). */
void oracle_qwen2_layer(const OracleQwen2* m, int l, float* h, void* kcache, void* vcache, int kv_f16,
                        int pos)
{
    h2f_init();
    const OracleQwen2Layer* L = &m->layer[l];
    const int H = m->hidden, F = m->ffn, hd = H / m->heads, qd = m->heads * hd, kvd = m->kv_heads * hd;
    const int S = m->max_seq, n = pos + 1;
    float* xn = (float*)malloc(sizeof(float) * (size_t)H);
    float* q = (float*)malloc(sizeof(float) * (size_t)qd);
    float* k = (float*)malloc(sizeof(float) * (size_t)kvd);
    float* v = (float*)malloc(sizeof(float) * (size_t)kvd);
    float* attn = (float*)malloc(sizeof(float) * (size_t)qd);
    float* o = (float*)malloc(sizeof(float) * (size_t)H);
    float* g = (float*)malloc(sizeof(float) * (size_t)F);
    float* u = (float*)malloc(sizeof(float) * (size_t)F);
    float* kf = (float*)malloc(sizeof(float) * (size_t)n * hd * m->kv_heads);
    float* vf = (float*)malloc(sizeof(float) * (size_t)n * hd * m->kv_heads);

    qwen2_rms_norm(h, L->attn_norm, xn, H, m->eps);
    oracle_mat_vec_f16(L->wq, H, xn, q, qd, H, L->bq, NULL);
    oracle_mat_vec_f16(L->wk, H, xn, k, kvd, H, L->bk, NULL);
    oracle_mat_vec_f16(L->wv, H, xn, v, kvd, H, L->bv, NULL);
    qwen2_rope(q, m->heads, hd, pos, m->rope_base);
    qwen2_rope(k, m->kv_heads, hd, pos, m->rope_base);

    for (int kvh = 0; kvh < m->kv_heads; ++kvh) {
        const size_t row = ((size_t)kvh * S + pos) * hd;
        for (int d = 0; d < hd; ++d) {
            if (kv_f16) {
                ((uint16_t*)kcache)[row + d] = oracle_f2h(k[kvh * hd + d]);
                ((uint16_t*)vcache)[row + d] = oracle_f2h(v[kvh * hd + d]);
            } else {
                ((float*)kcache)[row + d] = k[kvh * hd + d];
                ((float*)vcache)[row + d] = v[kvh * hd + d];
            }
        }
        for (int j = 0; j < n; ++j)
            for (int d = 0; d < hd; ++d) {
                const size_t src = ((size_t)kvh * S + j) * hd + d;
                const size_t dst = ((size_t)kvh * n + j) * hd + d;
                kf[dst] = kv_f16 ? h2f(((uint16_t*)kcache)[src]) : ((float*)kcache)[src];
                vf[dst] = kv_f16 ? h2f(((uint16_t*)vcache)[src]) : ((float*)vcache)[src];
            }
    }
    oracle_attention(q, kf, vf, attn, m->heads, m->kv_heads, n, hd, n * hd, 1.0f / sqrtf((float)hd));

    oracle_mat_vec_f16(L->wo, qd, attn, o, H, qd, NULL, NULL);
    for (int i = 0; i < H; ++i)
        h[i] = h[i] + o[i];
    qwen2_rms_norm(h, L->ffn_norm, xn, H, m->eps);
    oracle_mat_vec_f16(L->wgate, H, xn, g, F, H, NULL, NULL);
    oracle_mat_vec_f16(L->wup, H, xn, u, F, H, NULL, NULL);
    oracle_swiglu(g, u, g, F);
    oracle_mat_vec_f16(L->wdown, F, g, o, H, F, NULL, NULL);
    for (int i = 0; i < H; ++i)
        h[i] = h[i] + o[i];

    free(xn); free(q); free(k); free(v); free(attn); free(o); free(g); free(u); free(kf); free(vf);
}

/* One whole decode step: embed `token`, run every layer at `pos`, and write the logits. The
 * caches hold layers * kv_heads * max_seq * hd elements. Returns the greedy id. */
int oracle_qwen2_step(const OracleQwen2* m, void* kcache, void* vcache, int kv_f16, int token, int pos,
                      float* logits, float* hidden_out)
{
    h2f_init();
    const int H = m->hidden, hd = H / m->heads;
    const size_t per_layer = (size_t)m->kv_heads * m->max_seq * hd * (kv_f16 ? 2 : 4);
    float* h = (float*)malloc(sizeof(float) * (size_t)H);
    float* hn = (float*)malloc(sizeof(float) * (size_t)H);
    oracle_get_rows_f16(m->token_embd, H, token, h);
    for (int l = 0; l < m->layers; ++l)
        oracle_qwen2_layer(m, l, h, (char*)kcache + per_layer * l, (char*)vcache + per_layer * l, kv_f16, pos);
    qwen2_rms_norm(h, m->output_norm, hn, H, m->eps);
    oracle_mat_vec_f16(m->output, H, hn, logits, m->vocab, H, NULL, NULL);
    if (hidden_out)
        memcpy(hidden_out, h, sizeof(float) * (size_t)H);
    free(h);
    free(hn);
    return oracle_argmax(logits, m->vocab);
}

int oracle_num_threads(void) { return g_threads; }

void oracle_set_num_threads(int n)
{
    if (n > 0)
        g_threads = n;
}

/* ---- sampler (src/Sampler.cpp:10-98, src/Sampler.h:14-43) -------------------------------------
 * std::mt19937_64 restated from its published definition (Matsumoto & Nishimura, 64-bit MT):
 * n = 312, m = 156, r = 31, a = 0xB5026F5AA96619E9, tempering (u, d) = (29, 0x5555555555555555),
 * (s, b) = (17, 0x71D67FFFEDA60000), (t, c) = (37, 0xFFF7EEE000000000), l = 43, seeding multiplier
 * f = 6364136223846793005. */
typedef struct OracleMt64 {
    uint64_t mt[312];
    int idx;
} OracleMt64;

void oracle_mt64_seed(OracleMt64* s, uint64_t seed)
{
    s->mt[0] = seed;
    for (int i = 1; i < 312; ++i)
        s->mt[i] = 6364136223846793005ULL * (s->mt[i - 1] ^ (s->mt[i - 1] >> 62)) + (uint64_t)i;
    s->idx = 312;
}

uint64_t oracle_mt64_next(OracleMt64* s)
{
    const uint64_t upper = 0xFFFFFFFF80000000ULL, lower = 0x7FFFFFFFULL, a = 0xB5026F5AA96619E9ULL;
    if (s->idx >= 312) {
        for (int i = 0; i < 312; ++i) {
            const uint64_t x = (s->mt[i] & upper) | (s->mt[(i + 1) % 312] & lower);
            uint64_t xa = x >> 1;
            if (x & 1ULL)
                xa ^= a;
            s->mt[i] = s->mt[(i + 156) % 312] ^ xa;
        }
        s->idx = 0;
    }
    uint64_t y = s->mt[s->idx++];
    y ^= (y >> 29) & 0x5555555555555555ULL;
    y ^= (y << 17) & 0x71D67FFFEDA60000ULL;
    y ^= (y << 37) & 0xFFF7EEE000000000ULL;
    y ^= y >> 43;
    return y;
}

/* std::uniform_real_distribution<double>(0, 1) over a 64-bit engine: one draw x, x / 2^64 rounded
 * to double, and a value that rounds up to 1 is replaced by the largest double below 1. */
double oracle_mt64_canonical(OracleMt64* s)
{
    const double u = (double)oracle_mt64_next(s) * 0x1p-64;
    return u >= 1.0 ? nextafter(1.0, 0.0) : u;
}

static const float* g_sort_logits;
static int by_logit_desc(const void* pa, const void* pb)
{
    const int a = *(const int*)pa, b = *(const int*)pb;
    const float la = g_sort_logits[a], lb = g_sort_logits[b];
    if (la > lb)
        return -1;
    if (la < lb)
        return 1;
    return a < b ? -1 : (a > b);  /* equal logits: the lower index first */
}

/* Sampler::Sample. logits is modified in place (penalty, temperature), as the reference does. The
 * top-k order is by logit, then by index among equal logits (std::partial_sort leaves their order
 * unspecified). Not thread-safe (qsort's comparator reads a static). */
int oracle_sample(float* logits, int vocab, float temperature, int top_k, float top_p, float repeat_penalty,
                  int repeat_last_n, const int32_t* history, int hist_len, OracleMt64* rng)
{
    if (repeat_penalty != 1.0f && hist_len > 0) {  /* src/Sampler.cpp:12-29 */
        int begin = 0;
        if (repeat_last_n >= 0 && repeat_last_n < hist_len)
            begin = hist_len - repeat_last_n;
        for (int i = begin; i < hist_len; ++i) {
            const int t = history[i];
            if (t < 0 || t >= vocab)
                continue;
            const float v = logits[t];
            logits[t] = v > 0.0f ? v / repeat_penalty : v * repeat_penalty;
        }
    }
    if (temperature <= 0.0f) {  /* :31-41 greedy: the first index of the maximum */
        int best = 0;
        for (int i = 1; i < vocab; ++i)
            if (logits[i] > logits[best])
                best = i;
        return best;
    }
    for (int i = 0; i < vocab; ++i)  /* :43-46 */
        logits[i] /= temperature;
    const int k = top_k <= 0 ? vocab : (top_k < vocab ? top_k : vocab);  /* :48-55 */
    int* order = (int*)malloc(sizeof(int) * (size_t)vocab);
    double* w = (double*)malloc(sizeof(double) * (size_t)k);
    for (int i = 0; i < vocab; ++i)
        order[i] = i;
    g_sort_logits = logits;
    qsort(order, (size_t)vocab, sizeof(int), by_logit_desc);
    const float max_logit = logits[order[0]];  /* :57-64 */
    double total = 0.0;
    for (int i = 0; i < k; ++i) {
        w[i] = exp((double)(logits[order[i]] - max_logit));
        total += w[i];
    }
    int kept = k;  /* :66-77 nucleus */
    double cumulative = 0.0;
    for (int i = 0; i < k; ++i) {
        cumulative += w[i] / total;
        if (cumulative >= (double)top_p) {
            kept = i + 1;
            break;
        }
    }
    double kept_total = 0.0;
    for (int i = 0; i < kept; ++i)
        kept_total += w[i];
    const double target = oracle_mt64_canonical(rng) * kept_total;  /* :83-95 */
    double acc = 0.0;
    int token = order[kept - 1];
    for (int i = 0; i < kept; ++i) {
        acc += w[i];
        if (acc >= target) {
            token = order[i];
            break;
        }
    }
    free(order);
    free(w);
    return token;
}

size_t oracle_mt64_bytes(void) { return sizeof(OracleMt64); }
