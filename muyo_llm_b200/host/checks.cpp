// Run<Op>(): the reference's known-answer checks (src/<Op>.cpp) on the B200 kernels. Inputs and
// tolerances are the reference checks' own; the expected values come from plain CPU loops here.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "host.h"
#include "muyo_cuda.h"

namespace muyo_llm
{
namespace
{
void Check(int rc, const char* what)
{
    if (rc != MUYO_OK)
        throw std::runtime_error(std::string(what) + ": " + muyo_cuda_last_error());
}

void CudaCheck(cudaError_t e, const char* what)
{
    if (e != cudaSuccess)
        throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

/// A device copy of a host vector (or n zeroed elements), freed on scope exit.
template <typename T>
struct Dev {
    T* p = nullptr;
    size_t n = 0;
    explicit Dev(size_t count) : n(count)
    {
        CudaCheck(cudaMalloc(&p, sizeof(T) * (n ? n : 1)), "cudaMalloc");
        CudaCheck(cudaMemset(p, 0, sizeof(T) * (n ? n : 1)), "cudaMemset");
    }
    explicit Dev(const std::vector<T>& h) : Dev(h.size())
    {
        CudaCheck(cudaMemcpy(p, h.data(), sizeof(T) * n, cudaMemcpyHostToDevice), "cudaMemcpy H2D");
    }
    ~Dev() { cudaFree(p); }
    Dev(const Dev&) = delete;
    Dev& operator=(const Dev&) = delete;
    std::vector<T> Get() const
    {
        std::vector<T> h(n);
        CudaCheck(cudaDeviceSynchronize(), "kernel");
        CudaCheck(cudaMemcpy(h.data(), p, sizeof(T) * n, cudaMemcpyDeviceToHost), "cudaMemcpy D2H");
        return h;
    }
};

/// IEEE binary16 bits of f, rounded to nearest even (finite inputs of modest magnitude).
uint16_t ToHalf(float f)
{
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const int exp = (int)((x >> 23) & 0xff) - 127 + 15;
    uint32_t mant = x & 0x7fffffu;
    if (exp >= 31)
        return (uint16_t)(sign | 0x7c00u);
    if (exp <= 0) {  // subnormal or zero
        if (exp < -10)
            return (uint16_t)sign;
        mant |= 0x800000u;
        const int shift = 14 - exp;
        uint32_t h = mant >> shift;
        const uint32_t rem = mant & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u)))
            ++h;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)exp << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u)))
        ++h;  // a carry into the exponent is the correct rounding
    return (uint16_t)(sign | h);
}

float FromHalf(uint16_t h)
{
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const int exp = (h >> 10) & 0x1f;
    const uint32_t mant = h & 0x3ffu;
    float v;
    if (exp == 0)
        v = std::ldexp((float)mant, -24);
    else if (exp == 31)
        v = mant ? NAN : INFINITY;
    else
        v = std::ldexp((float)(mant | 0x400u), exp - 25);
    uint32_t bits;
    std::memcpy(&bits, &v, 4);
    bits |= sign;
    std::memcpy(&v, &bits, 4);
    return v;
}

/// |a - e| <= tol * (1 + |e|) for every element (src/TransformerLayer.cpp:602's form).
bool Close(const std::vector<float>& a, const std::vector<float>& e, double tol, const char* what)
{
    double worst = 0;
    size_t at = 0;
    bool ok = a.size() == e.size();
    for (size_t i = 0; ok && i < a.size(); ++i) {
        const double d = std::fabs((double)a[i] - e[i]) / (1.0 + std::fabs((double)e[i]));
        if (!(d <= tol))
            ok = false, at = i;
        if (d > worst)
            worst = d;
    }
    std::printf("[%s] %s (max rel err %.3g, tol %.3g)\n", what, ok ? "ok" : "MISMATCH", worst, tol);
    if (!ok && at < a.size())
        std::printf("[%s] first mismatch at %zu: got %.9g expected %.9g\n", what, at, a[at], e[at]);
    return ok;
}

MuyoBinaryParams Vec(uint32_t n)
{
    MuyoBinaryParams p{};
    p.ne = n;
    p.ne00 = p.ne10 = p.ne20 = n;
    p.ne01 = p.ne02 = p.ne03 = p.ne11 = p.ne12 = p.ne13 = p.ne21 = p.ne22 = p.ne23 = 1;
    p.nb00 = p.nb10 = p.nb20 = 1;
    p.nb01 = p.nb02 = p.nb03 = p.nb11 = p.nb12 = p.nb13 = p.nb21 = p.nb22 = p.nb23 = n;
    return p;
}

MuyoMatVecParams MatVec(uint32_t ncols, uint32_t rows)
{
    MuyoMatVecParams p{};
    p.ncols = p.stride_a = p.stride_b = ncols;
    p.stride_d = p.rows = rows;
    p.ne02 = p.ne12 = p.broadcast2 = p.broadcast3 = p.batches = 1;
    return p;
}

template <typename F>
int Guard(const char* what, F body)
{
    try {
        return body() ? 0 : 1;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "[%s] error: %s\n", what, e.what());
        return 1;
    }
}
}  // namespace

// src/ElementwiseAdd.cpp:93-99,209: a[i] = 0.5 i, b[i] = 1 + 0.25 i over 1000 elements, exact.
int RunElementwiseAdd()
{
    return Guard("add", [] {
        const uint32_t n = 1000;
        std::vector<float> a(n), b(n), e(n);
        for (uint32_t i = 0; i < n; ++i)
            a[i] = 0.5F * (float)i, b[i] = 1.0F + 0.25F * (float)i, e[i] = a[i] + b[i];
        Dev<float> da(a), db(b), dd(n);
        const MuyoBinaryParams p = Vec(n);
        Check(muyo_cuda_add(&p, da.p, db.p, dd.p, nullptr), "add");
        return Close(dd.Get(), e, 0.0, "add");
    });
}

// src/MatVec.cpp:68-80,202: W[r][c] = (c % 7) - 3 (F16), x[c] = (c % 5) - 2, 128 x 256, exact.
int RunMatVec()
{
    return Guard("matvec", [] {
        const uint32_t rows = 128, cols = 256;
        std::vector<uint16_t> w((size_t)rows * cols);
        std::vector<float> x(cols), e(rows, 0.0F);
        for (uint32_t c = 0; c < cols; ++c)
            x[c] = (float)((int)(c % 5) - 2);
        for (uint32_t r = 0; r < rows; ++r)
            for (uint32_t c = 0; c < cols; ++c) {
                const float v = (float)((int)(c % 7) - 3);
                w[(size_t)r * cols + c] = ToHalf(v);
                e[r] += v * x[c];
            }
        Dev<uint16_t> dw(w);
        Dev<float> dx(x), dy(rows);
        const MuyoMatVecParams p = MatVec(cols, rows);
        Check(muyo_cuda_mat_vec_f16(&p, dw.p, dx.p, dy.p, nullptr, nullptr, nullptr), "mat_vec_f16");
        return Close(dy.Get(), e, 0.0, "matvec");
    });
}

// src/RmsNorm.cpp:41-72: 8 rows of 512, x = ((r*512 + c) % 13) - 6, w = 0.5 + 0.001 (c % 11),
// eps 1e-6, tol 1e-4.
int RunRmsNorm()
{
    return Guard("rmsnorm", [] {
        const uint32_t rows = 8, n = 512;
        std::vector<float> x((size_t)rows * n), w(n), e(x.size());
        for (uint32_t c = 0; c < n; ++c)
            w[c] = 0.5F + 0.001F * (float)(c % 11);
        for (uint32_t r = 0; r < rows; ++r) {
            double ss = 0;
            for (uint32_t c = 0; c < n; ++c) {
                const float v = (float)((int)((r * n + c) % 13) - 6);
                x[(size_t)r * n + c] = v;
                ss += (double)v * v;
            }
            const double scale = 1.0 / std::sqrt(ss / n + 1e-6);
            for (uint32_t c = 0; c < n; ++c)
                e[(size_t)r * n + c] = (float)(x[(size_t)r * n + c] * scale * w[c]);
        }
        Dev<float> dx(x), dw(w), dd(x.size());
        MuyoBinaryParams p{};
        p.ne = rows * n;
        p.ne00 = p.ne20 = n, p.ne01 = p.ne21 = rows, p.ne02 = p.ne03 = p.ne22 = p.ne23 = 1;
        p.nb00 = p.nb20 = 1, p.nb01 = p.nb21 = n, p.nb02 = p.nb03 = p.nb22 = p.nb23 = n * rows;
        p.ne10 = n, p.ne11 = p.ne12 = p.ne13 = 1, p.nb10 = 1;
        p.param1 = 1e-6F;
        Check(muyo_cuda_rms_norm(&p, dx.p, dw.p, dd.p, nullptr), "rms_norm");
        return Close(dd.Get(), e, 1e-4, "rmsnorm");
    });
}

// src/Rope.cpp:41-64,204: one NEOX row of 8 channels c - 3 at position 3, base 1e4, tol 1e-5.
int RunRope()
{
    return Guard("rope", [] {
        const uint32_t hd = 8;
        const int pos = 3;
        std::vector<float> x(hd), e(hd);
        for (uint32_t c = 0; c < hd; ++c)
            x[c] = (float)c - 3.0F;
        const float theta_scale = std::pow(10000.0F, -2.0F / (float)hd);
        for (uint32_t j = 0; j < hd / 2; ++j) {
            const float th = (float)pos * std::pow(theta_scale, (float)j);
            e[j] = x[j] * std::cos(th) - x[j + hd / 2] * std::sin(th);
            e[j + hd / 2] = x[j] * std::sin(th) + x[j + hd / 2] * std::cos(th);
        }
        Dev<float> dx(x), dd(hd);
        Dev<int32_t> dp(std::vector<int32_t>{pos});
        MuyoRopeParams p{};
        p.rope_mode = MUYO_ROPE_NEOX;
        p.nrows = 1, p.n_dims = hd, p.n_offs = 0;
        p.freq_scale = 1.0F, p.freq_base = 10000.0F, p.attn_factor = 1.0F, p.theta_scale = theta_scale;
        p.ne00 = hd, p.ne01 = 1, p.ne02 = 1, p.nb01 = hd, p.nb11 = hd;
        Check(muyo_cuda_rope(&p, dx.p, dp.p, nullptr, dd.p, nullptr), "rope");
        return Close(dd.Get(), e, 1e-5, "rope");
    });
}

// src/Swiglu.cpp:42,60-67,188: g = 0.01 ((i % 17) - 8), u = 0.5 + 0.01 (i % 7), 600 elements, tol 1e-5.
int RunSwiglu()
{
    return Guard("swiglu", [] {
        const uint32_t n = 600;
        std::vector<float> g(n), u(n), e(n);
        for (uint32_t i = 0; i < n; ++i) {
            g[i] = 0.01F * (float)((int)(i % 17) - 8), u[i] = 0.5F + 0.01F * (float)(i % 7);
            e[i] = (float)(g[i] / (1.0 + std::exp(-(double)g[i])) * u[i]);
        }
        Dev<float> dg(g), du(u), dd(n);
        MuyoGluParams p{};
        p.N = n, p.ne00 = n, p.ne20 = n, p.mode = MUYO_GLU_SPLIT;
        p.nb00 = p.nb10 = p.nb20 = 1;
        p.nb01 = p.nb11 = p.nb21 = n, p.nb02 = p.nb03 = p.nb12 = p.nb13 = p.nb22 = p.nb23 = n;
        p.ne21 = p.ne22 = 1;
        Check(muyo_cuda_swiglu(&p, dg.p, du.p, dd.p, nullptr), "swiglu");
        return Close(dd.Get(), e, 1e-5, "swiglu");
    });
}

// src/GetRows.cpp:40-55,182: table[t][c] = (t % 5) - 2 + 0.001 c (1024 x 512), token 7, exact.
int RunGetRows()
{
    return Guard("getrows", [] {
        const uint32_t vocab = 1024, n = 512;
        const int32_t token = 7;
        std::vector<float> t((size_t)vocab * n), e(n);
        for (uint32_t r = 0; r < vocab; ++r)
            for (uint32_t c = 0; c < n; ++c)
                t[(size_t)r * n + c] = (float)((int)(r % 5) - 2) + 0.001F * (float)c;
        for (uint32_t c = 0; c < n; ++c)
            e[c] = t[(size_t)token * n + c];
        Dev<float> dt(t), dd(n);
        Dev<int32_t> di(std::vector<int32_t>{token});
        MuyoBinaryParams p{};
        p.ne = n;
        p.ne00 = n, p.ne01 = vocab, p.ne02 = p.ne03 = 1, p.nb00 = 1, p.nb01 = n, p.nb02 = p.nb03 = n * vocab;
        p.ne10 = 1, p.ne11 = p.ne12 = p.ne13 = 1, p.nb10 = 1, p.nb11 = p.nb12 = p.nb13 = 1;
        p.ne20 = n, p.ne21 = p.ne22 = p.ne23 = 1, p.nb20 = 1, p.nb21 = p.nb22 = p.nb23 = n;
        Check(muyo_cuda_get_rows_f32(&p, dt.p, di.p, dd.p, nullptr), "get_rows_f32");
        return Close(dd.Get(), e, 0.0, "getrows");
    });
}

// src/Argmax.cpp:41-56,146: x[i] = -1 + 0.001 i over 32, x[21] = 5 -> 21.
int RunArgmax()
{
    return Guard("argmax", [] {
        const uint32_t n = 32;
        std::vector<float> x(n);
        for (uint32_t i = 0; i < n; ++i)
            x[i] = -1.0F + 0.001F * (float)i;
        x[21] = 5.0F;
        MuyoGenericParams p{n, 1, 0, 0, 0, 0};
        const size_t ws = muyo_cuda_argmax_workspace_size(&p);
        Dev<float> dx(x);
        Dev<int32_t> dd(1);
        Dev<unsigned char> dws(ws);
        Check(muyo_cuda_argmax(&p, dx.p, dd.p, dws.p, ws, nullptr), "argmax");
        const int32_t got = dd.Get()[0];
        std::printf("[argmax] %s (got %d, expected 21)\n", got == 21 ? "ok" : "MISMATCH", got);
        return got == 21;
    });
}

// src/SoftMax.cpp:42-55,183: one row of 64, x = (c % 9) - 4, scale 1/8, tol 1e-5.
int RunSoftMax()
{
    return Guard("softmax", [] {
        const uint32_t n = 64;
        const float scale = 0.125F;
        std::vector<float> x(n), e(n);
        double mx = -1e300, sum = 0;
        for (uint32_t c = 0; c < n; ++c)
            x[c] = (float)((int)(c % 9) - 4), mx = std::fmax(mx, (double)x[c] * scale);
        for (uint32_t c = 0; c < n; ++c)
            sum += std::exp((double)x[c] * scale - mx);
        for (uint32_t c = 0; c < n; ++c)
            e[c] = (float)(std::exp((double)x[c] * scale - mx) / sum);
        Dev<float> dx(x), dd(n);
        MuyoSoftMaxParams p{};
        p.KX = n, p.ne00 = n, p.ne01 = 1, p.ne02 = p.ne12 = p.ne13 = 1, p.scale = scale, p.nrows_x = 1;
        Check(muyo_cuda_soft_max(&p, dx.p, nullptr, nullptr, dd.p, nullptr), "soft_max");
        return Close(dd.Get(), e, 1e-5, "softmax");
    });
}

// src/Attention.cpp:42-105,286: head_dim 8, 16 keys; q[d] = (d % 5) - 2, K[k][d] = ((k + d) % 3) - 1,
// V[k][d] = ((2k + d) % 7) - 3; scores GEMV -> soft_max (scale 1/sqrt(8)) -> values GEMV over the
// transposed V, the reference's three-node chain; tol 1e-4.
int RunAttention()
{
    return Guard("attention", [] {
        const uint32_t hd = 8, nk = 16;
        const float scale = 1.0F / std::sqrt((float)hd);
        std::vector<float> q(hd), K((size_t)nk * hd), Vt((size_t)hd * nk), e(hd, 0.0F);
        for (uint32_t d = 0; d < hd; ++d)
            q[d] = (float)((int)(d % 5) - 2);
        for (uint32_t k = 0; k < nk; ++k)
            for (uint32_t d = 0; d < hd; ++d) {
                K[(size_t)k * hd + d] = (float)((int)((k + d) % 3) - 1);
                Vt[(size_t)d * nk + k] = (float)((int)((k * 2 + d) % 7) - 3);
            }
        std::vector<double> pr(nk);
        double mx = -1e300, sum = 0;
        for (uint32_t k = 0; k < nk; ++k) {
            double s = 0;
            for (uint32_t d = 0; d < hd; ++d)
                s += (double)q[d] * K[(size_t)k * hd + d];
            pr[k] = s * scale, mx = std::fmax(mx, pr[k]);
        }
        for (uint32_t k = 0; k < nk; ++k)
            pr[k] = std::exp(pr[k] - mx), sum += pr[k];
        for (uint32_t d = 0; d < hd; ++d) {
            double o = 0;
            for (uint32_t k = 0; k < nk; ++k)
                o += pr[k] / sum * Vt[(size_t)d * nk + k];
            e[d] = (float)o;
        }
        Dev<float> dq(q), dk(K), dvt(Vt), ds(nk), dp(nk), dout(hd);
        const MuyoMatVecParams ps = MatVec(hd, nk), pv = MatVec(nk, hd);
        MuyoSoftMaxParams sm{};
        sm.KX = nk, sm.ne00 = nk, sm.ne01 = 1, sm.ne02 = sm.ne12 = sm.ne13 = 1, sm.scale = scale, sm.nrows_x = 1;
        Check(muyo_cuda_mat_vec_f32(&ps, dk.p, dq.p, ds.p, nullptr, nullptr, nullptr), "scores");
        Check(muyo_cuda_soft_max(&sm, ds.p, nullptr, nullptr, dp.p, nullptr), "soft_max");
        Check(muyo_cuda_mat_vec_f32(&pv, dvt.p, dp.p, dout.p, nullptr, nullptr, nullptr), "values");
        return Close(dout.Get(), e, 1e-4, "attention");
    });
}

// src/KvCache.cpp:40-44,356-406: one head of 16, cache of 4 positions, two tokens appended (key
// rotated by NEOX RoPE, base 1e4, at its position) and attended over; tol 1e-4. The key/value/query
// patterns are small integers as in the reference check.
int RunKvCache()
{
    return Guard("kvcache", [] {
        const uint32_t hd = 16, max_seq = 4, tokens = 2;
        const double base = 10000.0;
        std::vector<float> kc((size_t)max_seq * hd, 0.0F), vc((size_t)max_seq * hd, 0.0F);
        Dev<float> dkc(kc), dvc(vc), dout(hd);
        MuyoAttentionParams ap{1, 1, hd, max_seq, 0, MUYO_KV_F32, 1.0F / std::sqrt((float)hd)};
        const size_t ws = muyo_cuda_attention_workspace_size(&ap);
        Dev<unsigned char> dws(ws);
        bool ok = true;
        for (uint32_t t = 0; t < tokens; ++t) {
            std::vector<float> k(hd), v(hd), q(hd);
            for (uint32_t d = 0; d < hd; ++d) {
                k[d] = (float)((int)((d + 3 * t) % 5) - 2);
                v[d] = (float)((int)((2 * d + t) % 7) - 3);
                q[d] = (float)((int)((d + t) % 4) - 1);
            }
            // expected: rotate k at position t, append, attend q over keys 0..t
            for (uint32_t j = 0; j < hd / 2; ++j) {
                const double th = (double)t * std::pow(base, -2.0 * j / hd);
                const double c = std::cos(th), s = std::sin(th);
                kc[(size_t)t * hd + j] = (float)(k[j] * c - k[j + hd / 2] * s);
                kc[(size_t)t * hd + j + hd / 2] = (float)(k[j] * s + k[j + hd / 2] * c);
            }
            for (uint32_t d = 0; d < hd; ++d)
                vc[(size_t)t * hd + d] = v[d];
            std::vector<double> pr(t + 1);
            double mx = -1e300, sum = 0;
            for (uint32_t i = 0; i <= t; ++i) {
                double sc = 0;
                for (uint32_t d = 0; d < hd; ++d)
                    sc += (double)q[d] * kc[(size_t)i * hd + d];
                pr[i] = sc * ap.scale, mx = std::fmax(mx, pr[i]);
            }
            for (uint32_t i = 0; i <= t; ++i)
                pr[i] = std::exp(pr[i] - mx), sum += pr[i];
            std::vector<float> e(hd);
            for (uint32_t d = 0; d < hd; ++d) {
                double o = 0;
                for (uint32_t i = 0; i <= t; ++i)
                    o += pr[i] / sum * vc[(size_t)i * hd + d];
                e[d] = (float)o;
            }
            Dev<float> dk(k), dv(v), dq(q);
            Dev<int32_t> dpos(std::vector<int32_t>{(int32_t)t});
            Check(muyo_cuda_kv_append(&ap, (float)base, dk.p, dv.p, dkc.p, dvc.p, dpos.p, nullptr), "kv_append");
            Check(muyo_cuda_attention_decode(&ap, dq.p, dkc.p, dvc.p, dpos.p, dout.p, dws.p, ws, nullptr),
                  "attention_decode");
            const std::string what = "kvcache token " + std::to_string(t);
            ok = Close(dout.Get(), e, 1e-4, what.c_str()) && ok;
        }
        return ok;
    });
}

// src/TransformerLayer.cpp's check itself: its inputs (:257-286: hidden 64, 8 cached keys, feed-forward
// 128, F32 weights in small integer patterns, position 0) through its 14 nodes as the op-level entry
// points (rms_norm, mat_vec_f32, rope_neox, mat_vec_f32, soft_max, mat_vec_f32, mat_vec_f32, add,
// rms_norm, mat_vec_f32 x2, swiglu, mat_vec_f32, add), against the same CPU sequence (:537-590) at the
// check's tolerance 1e-3 * (1 + |e|) (:602).
static bool ReferenceLayerChain()
{
    const uint32_t H = 64, S = 8, F = 128;
    const float eps = 1e-6F, scale = 1.0F / 8.0F;
    std::vector<float> hidden(H), n1(H), n2(H), wq((size_t)H * H), wo((size_t)H * H), wg((size_t)F * H),
        wu((size_t)F * H), wd((size_t)H * F), keys((size_t)S * H), vt((size_t)H * S);
    for (uint32_t i = 0; i < H; ++i) {
        hidden[i] = (float)((int)(i % 7) - 3);
        n1[i] = 0.5F + 0.01F * (float)(i % 5);
        n2[i] = 0.6F + 0.01F * (float)(i % 3);
    }
    for (uint32_t i = 0; i < H * H; ++i) {
        wq[i] = (float)((int)(i % 3) - 1);
        wo[i] = (float)((int)(i % 5) - 2) * 0.5F;
    }
    for (uint32_t i = 0; i < F * H; ++i) {
        wg[i] = (float)((int)(i % 3) - 1);
        wu[i] = (float)((int)(i % 4) - 1);
    }
    for (uint32_t i = 0; i < H * F; ++i)
        wd[i] = (float)((int)(i % 5) - 2) * 0.25F;
    for (uint32_t k = 0; k < S; ++k)
        for (uint32_t d = 0; d < H; ++d) {
            keys[(size_t)k * H + d] = (float)((int)((k + d) % 3) - 1);
            vt[(size_t)d * S + k] = (float)((int)((k * 2 + d) % 7) - 3);
        }
    // CPU sequence (float sums as the check's Gemv; double sum of squares as its RmsNorm)
    auto gemv = [](const std::vector<float>& w, const std::vector<float>& x, uint32_t rows) {
        std::vector<float> y(rows);
        for (uint32_t r = 0; r < rows; ++r) {
            float s = 0.0F;
            for (size_t k = 0; k < x.size(); ++k)
                s += w[r * x.size() + k] * x[k];
            y[r] = s;
        }
        return y;
    };
    auto norm = [&](const std::vector<float>& x, const std::vector<float>& w) {
        double ss = 0.0;
        for (float v : x)
            ss += (double)v * v;
        const float sc = (float)(1.0 / std::sqrt(ss / x.size() + eps));
        std::vector<float> y(x.size());
        for (size_t i = 0; i < x.size(); ++i)
            y[i] = x[i] * sc * w[i];
        return y;
    };
    const std::vector<float> xn = norm(hidden, n1), q = gemv(wq, xn, H);
    std::vector<float> qr(q);  // position 0: the rotation is the identity (cos 0 = 1, sin 0 = 0)
    const std::vector<float> sc = gemv(keys, qr, S);
    float mx = -1e30F;
    for (float v : sc)
        mx = std::max(mx, v * scale);
    std::vector<float> pr(S);
    double sum = 0.0;
    for (uint32_t k = 0; k < S; ++k)
        pr[k] = std::exp(sc[k] * scale - mx), sum += pr[k];
    for (float& v : pr)
        v = (float)(v / sum);
    const std::vector<float> o = gemv(wo, gemv(vt, pr, H), H);
    std::vector<float> x1(H);
    for (uint32_t i = 0; i < H; ++i)
        x1[i] = hidden[i] + o[i];
    const std::vector<float> xn2 = norm(x1, n2), g = gemv(wg, xn2, F), u = gemv(wu, xn2, F);
    std::vector<float> act(F);
    for (uint32_t i = 0; i < F; ++i)
        act[i] = g[i] / (1.0F + std::exp(-g[i])) * u[i];
    const std::vector<float> mlp = gemv(wd, act, H);
    std::vector<float> e(H);
    for (uint32_t i = 0; i < H; ++i)
        e[i] = x1[i] + mlp[i];
    // device: the 14 nodes
    Dev<float> dh(hidden), dn1(n1), dn2(n2), dwq(wq), dwo(wo), dwg(wg), dwu(wu), dwd(wd), dk(keys), dvt(vt);
    Dev<float> dxn(H), dq(H), dqr(H), dsc(S), dpr(S), datt(H), dout1(H), dx1(H), dxn2(H), dg(F), du(F), dact(F),
        dmlp(H), dy(H);
    Dev<int32_t> dpos(std::vector<int32_t>{0});
    MuyoBinaryParams pn = Vec(H);
    pn.param1 = eps;
    MuyoRopeParams pr_{};
    pr_.rope_mode = MUYO_ROPE_NEOX, pr_.nrows = 1, pr_.n_dims = H, pr_.n_offs = 0;
    pr_.freq_scale = 1.0F, pr_.freq_base = 10000.0F, pr_.attn_factor = 1.0F;
    pr_.theta_scale = std::pow(10000.0F, -2.0F / (float)H);
    pr_.ne00 = H, pr_.ne01 = 1, pr_.ne02 = 1, pr_.nb01 = H, pr_.nb11 = H;
    MuyoSoftMaxParams psm{};
    psm.KX = S, psm.ne00 = S, psm.ne01 = 1, psm.ne02 = psm.ne12 = psm.ne13 = 1, psm.scale = scale, psm.nrows_x = 1;
    MuyoGluParams pg{};
    pg.N = F, pg.ne00 = F, pg.ne20 = F, pg.mode = MUYO_GLU_SPLIT;
    pg.nb00 = pg.nb10 = pg.nb20 = 1;
    pg.nb01 = pg.nb11 = pg.nb21 = F, pg.nb02 = pg.nb03 = pg.nb12 = pg.nb13 = pg.nb22 = pg.nb23 = F;
    pg.ne21 = pg.ne22 = 1;
    const MuyoMatVecParams mhh = MatVec(H, H), mhs = MatVec(H, S), msh = MatVec(S, H), mhf = MatVec(H, F),
                           mfh = MatVec(F, H);
    const MuyoBinaryParams pa = Vec(H);
    Check(muyo_cuda_rms_norm(&pn, dh.p, dn1.p, dxn.p, nullptr), "PreNorm");
    Check(muyo_cuda_mat_vec_f32(&mhh, dwq.p, dxn.p, dq.p, nullptr, nullptr, nullptr), "QProj");
    Check(muyo_cuda_rope(&pr_, dq.p, dpos.p, nullptr, dqr.p, nullptr), "QRope");
    Check(muyo_cuda_mat_vec_f32(&mhs, dk.p, dqr.p, dsc.p, nullptr, nullptr, nullptr), "AttnScores");
    Check(muyo_cuda_soft_max(&psm, dsc.p, nullptr, nullptr, dpr.p, nullptr), "AttnWeights");
    Check(muyo_cuda_mat_vec_f32(&msh, dvt.p, dpr.p, datt.p, nullptr, nullptr, nullptr), "AttnOut");
    Check(muyo_cuda_mat_vec_f32(&mhh, dwo.p, datt.p, dout1.p, nullptr, nullptr, nullptr), "OProj");
    Check(muyo_cuda_add(&pa, dh.p, dout1.p, dx1.p, nullptr), "Residual1");
    Check(muyo_cuda_rms_norm(&pn, dx1.p, dn2.p, dxn2.p, nullptr), "PostNorm");
    Check(muyo_cuda_mat_vec_f32(&mhf, dwg.p, dxn2.p, dg.p, nullptr, nullptr, nullptr), "GateProj");
    Check(muyo_cuda_mat_vec_f32(&mhf, dwu.p, dxn2.p, du.p, nullptr, nullptr, nullptr), "UpProj");
    Check(muyo_cuda_swiglu(&pg, dg.p, du.p, dact.p, nullptr), "SwiGLU");
    Check(muyo_cuda_mat_vec_f32(&mfh, dwd.p, dact.p, dmlp.p, nullptr, nullptr, nullptr), "DownProj");
    Check(muyo_cuda_add(&pa, dx1.p, dmlp.p, dy.p, nullptr), "Residual2");
    return Close(dy.Get(), e, 1e-3, "layer (the reference check's 14 nodes)");
}

// The decode step's fused layer (muyo_cuda_layer_step, five kernels) on a small Qwen2 layer with the
// same sizes: one head of 64, F32 cache, positions 0..7 decoded in turn, every output compared with a
// CPU restatement of the layer.
static bool FusedLayerSteps()
{
    {
        const uint32_t H = 64, F = 128, S = 8, hd = 64;
        const float eps = 1e-6F, base = 10000.0F;
        auto pat = [](uint32_t i, uint32_t m, float s) { return s * (float)((int)((i * 37u + 11u) % m) - (int)(m / 2)); };
        std::vector<float> n1(H), n2(H), bqkv(3 * H);
        std::vector<float> wqkv((size_t)3 * H * H), wo((size_t)H * H), wg((size_t)F * H), wu((size_t)F * H),
            wd((size_t)H * F);
        for (uint32_t i = 0; i < H; ++i)
            n1[i] = 1.0F + pat(i, 7, 0.01F), n2[i] = 1.0F + pat(i + 3, 5, 0.01F);
        for (uint32_t i = 0; i < 3 * H; ++i)
            bqkv[i] = pat(i, 9, 0.01F);
        auto fill16 = [&](std::vector<float>& w, uint32_t salt) {
            std::vector<uint16_t> h(w.size());
            for (size_t i = 0; i < w.size(); ++i) {
                h[i] = ToHalf(pat((uint32_t)i + salt, 17, 0.004F));
                w[i] = FromHalf(h[i]);
            }
            return h;
        };
        const auto hqkv = fill16(wqkv, 1), ho = fill16(wo, 2), hg = fill16(wg, 3), hu = fill16(wu, 4),
                   hdn = fill16(wd, 5);
        Dev<float> dn1(n1), dn2(n2), db(bqkv);
        Dev<uint16_t> dqkv(hqkv), dwo(ho), dwg(hg), dwu(hu), dwd(hdn);
        Dev<float> dkc((size_t)S * hd), dvc((size_t)S * hd), dx(H), dy(H);
        MuyoQwen2Config cfg{1, H, F, 1, 1, 0, S, eps, base, MUYO_KV_F32};
        const size_t ws = muyo_cuda_layer_workspace_size(&cfg);
        Dev<unsigned char> dws(ws + 256);
        void* wsp = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(dws.p) + 255) & ~uintptr_t(255));
        const MuyoLayerWeights lw{dn1.p, dqkv.p, db.p, dwo.p, dn2.p, dwg.p, dwu.p, dwd.p};

        std::vector<float> kc((size_t)S * hd), vc((size_t)S * hd);
        auto norm = [&](const std::vector<float>& x, const std::vector<float>& w) {
            double ss = 0;
            for (float v : x)
                ss += (double)v * v;
            const double s = std::sqrt(ss / x.size() + eps);
            std::vector<float> y(x.size());
            for (size_t i = 0; i < x.size(); ++i)
                y[i] = (float)(x[i] / s * w[i]);
            return y;
        };
        auto gemv = [](const std::vector<float>& w, const std::vector<float>& x, size_t rows) {
            std::vector<float> y(rows);
            for (size_t r = 0; r < rows; ++r) {
                double s = 0;
                for (size_t c = 0; c < x.size(); ++c)
                    s += (double)w[r * x.size() + c] * x[c];
                y[r] = (float)s;
            }
            return y;
        };
        auto rope = [&](float* v, uint32_t pos) {
            for (uint32_t j = 0; j < hd / 2; ++j) {
                const double th = (double)pos * std::pow((double)base, -2.0 * j / hd);
                const double c = std::cos(th), s = std::sin(th), a = v[j], b = v[j + hd / 2];
                v[j] = (float)(a * c - b * s), v[j + hd / 2] = (float)(a * s + b * c);
            }
        };
        bool ok = true;
        for (uint32_t pos = 0; pos < S; ++pos) {
            std::vector<float> x(H);
            for (uint32_t i = 0; i < H; ++i)
                x[i] = pat(i + 7 * pos, 13, 0.1F);
            // CPU restatement of the layer
            std::vector<float> qkv = gemv(wqkv, norm(x, n1), 3 * H);
            for (uint32_t i = 0; i < 3 * H; ++i)
                qkv[i] += bqkv[i];
            rope(qkv.data(), pos);
            rope(qkv.data() + H, pos);
            std::copy(qkv.begin() + H, qkv.begin() + 2 * H, kc.begin() + (size_t)pos * hd);
            std::copy(qkv.begin() + 2 * H, qkv.end(), vc.begin() + (size_t)pos * hd);
            std::vector<double> pr(pos + 1);
            double mx = -1e300, sum = 0;
            for (uint32_t t = 0; t <= pos; ++t) {
                double s = 0;
                for (uint32_t d = 0; d < hd; ++d)
                    s += (double)qkv[d] * kc[(size_t)t * hd + d];
                pr[t] = s / std::sqrt((double)hd), mx = std::fmax(mx, pr[t]);
            }
            for (uint32_t t = 0; t <= pos; ++t)
                pr[t] = std::exp(pr[t] - mx), sum += pr[t];
            std::vector<float> att(hd);
            for (uint32_t d = 0; d < hd; ++d) {
                double o = 0;
                for (uint32_t t = 0; t <= pos; ++t)
                    o += pr[t] / sum * vc[(size_t)t * hd + d];
                att[d] = (float)o;
            }
            std::vector<float> h1 = gemv(wo, att, H);
            for (uint32_t i = 0; i < H; ++i)
                h1[i] += x[i];
            const std::vector<float> hn = norm(h1, n2);
            const std::vector<float> g = gemv(wg, hn, F), u = gemv(wu, hn, F);
            std::vector<float> act(F);
            for (uint32_t i = 0; i < F; ++i)
                act[i] = (float)(g[i] / (1.0 + std::exp(-(double)g[i])) * u[i]);
            std::vector<float> e = gemv(wd, act, H);
            for (uint32_t i = 0; i < H; ++i)
                e[i] += h1[i];
            // device
            CudaCheck(cudaMemcpy(dx.p, x.data(), sizeof(float) * H, cudaMemcpyHostToDevice), "x");
            Dev<int32_t> dpos(std::vector<int32_t>{(int32_t)pos});
            Check(muyo_cuda_layer_step(&cfg, &lw, dkc.p, dvc.p, dpos.p, dx.p, dy.p, wsp, ws, nullptr), "layer_step");
            const std::string what = "layer pos " + std::to_string(pos);
            ok = Close(dy.Get(), e, 1e-3, what.c_str()) && ok;
        }
        return ok;
    }
}

int RunTransformerLayer()
{
    return Guard("layer", [] {
        const bool a = ReferenceLayerChain();
        const bool b = FusedLayerSteps();
        return a && b;
    });
}
}  // namespace muyo_llm
