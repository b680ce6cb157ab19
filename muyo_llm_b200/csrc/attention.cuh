// Split-K GQA decode attention over the persistent KV cache (flash-decoding style).
//
// Work item (kv head, 64-key chunk): the item stages its K and V tiles in shared memory once (F16 or
// F32 cache, converted to F32) and serves all `gqa` query heads of the group from them, which is the
// GQA broadcast of tools/reference_qwen2.py:133 and shaders/llama/mul_mat_vec_base.glsl:55-64
// without re-reading K/V per query head. Each item writes (max, sum, unnormalised output) per query
// head; the chunks are merged by the last CTA of the KV head to finish (a self-resetting arrival
// counter, the fused layer step), by a separate combine kernel (the op-level entry point, whose
// workspace may hold anything), or by the consumer of the output (the persistent decode kernel).
//
// With FUSED the item also performs the step's KV append: it rotates the raw key with NeoX RoPE in
// double precision (theta = pos * base^(-2j/hd), the rotation of tools/reference_qwen2.py:84-93,
// evaluated in float64 as there and rounded once), rounds key and value to the cache type, and the
// item holding the last chunk stores them at row `pos`; that item also uses the stored values for
// key `pos` itself, so every item reads only rows that earlier steps finished writing.
//
// All loads of data written on the device go through L2 (ld.global.cg): in the persistent kernel the
// producer of a row can be another SM within the same launch.
#pragma once

#include "common.cuh"

namespace muyo {

constexpr int kAttnKeys = 64;      // keys per work item
constexpr int kAttnThreads = 512;  // threads of the standalone attention CTA
constexpr int kAttnMaxGroup = 16;  // query heads per KV head

struct AttnDev {
    int heads, kv_heads, gqa, max_seq, n_keys_fixed;
    float scale;
    double rope_base;
    int max_chunks;
    const double* rope_cs;  // optional [max_seq][hd]: cos theta_j at [pos*hd + j], sin at [pos*hd + hd/2 + j]
};

template <typename KV>
__device__ __forceinline__ float kv_load(const KV* p);
template <>
__device__ __forceinline__ float kv_load<float>(const float* p)
{
    return __ldcg(p);
}
template <>
__device__ __forceinline__ float kv_load<__half>(const __half* p)
{
    return __half2float(__ldcg(p));
}

template <typename KV>
__device__ __forceinline__ KV kv_round(float v);
template <>
__device__ __forceinline__ float kv_round<float>(float v)
{
    return v;
}
template <>
__device__ __forceinline__ __half kv_round<__half>(float v)
{
    return __float2half_rn(v);
}

template <typename KV>
__device__ __forceinline__ float kv_value(KV v);
template <>
__device__ __forceinline__ float kv_value<float>(float v)
{
    return v;
}
template <>
__device__ __forceinline__ float kv_value<__half>(__half v)
{
    return __half2float(v);
}

// Rotated pair, as numpy computes x[:half]*c - x[half:]*s and x[:half]*s + x[half:]*c in float64
// from float32 inputs: products and sums rounded to double without contraction, one rounding to
// float at the end.
__device__ __forceinline__ void rope_pair_f64(float x0, float x1, double c, double s, float& y0, float& y1)
{
    y0 = __double2float_rn(__dsub_rn(__dmul_rn((double)x0, c), __dmul_rn((double)x1, s)));
    y1 = __double2float_rn(__dadd_rn(__dmul_rn((double)x0, s), __dmul_rn((double)x1, c)));
}

__device__ __forceinline__ void rope_cs_f64(int pos, int j, int hd, double base, double& c, double& s)
{
    const double theta = (double)pos * pow(base, -2.0 * (double)j / (double)hd);
    c = cos(theta);
    s = sin(theta);
}

// Shared-memory footprint of one work item (floats), excluding the double cos/sin table (hd doubles).
__host__ __device__ constexpr int attn_smem_floats(int hd, int g)
{
    return 2 * kAttnKeys * (hd + 1) /* K, V tiles */ + g * hd /* q */ + g * kAttnKeys /* p */ + 2 * g /* m, l */ +
           2 * hd /* new k, v */;
}

// part layout per (kv head, chunk, group member): [m, l, o[0..hd)]
template <int HD>
__device__ __forceinline__ float* part_ptr(float* part, const AttnDev& p, int kvh, int chunk, int g)
{
    return part + ((size_t)(kvh * p.max_chunks + chunk) * p.gqa + g) * (HD + 2);
}

// Merge of one output element (query head h = kvh*gqa + g, channel d) over nchunks partials.
template <int HD>
__device__ __forceinline__ float attn_merge_one(const AttnDev& p, const float* part, int kvh, int g, int d,
                                                int nchunks)
{
    float M = -INFINITY;
    for (int c = 0; c < nchunks; ++c)
        M = fmaxf(M, __ldcg(part_ptr<HD>(const_cast<float*>(part), p, kvh, c, g)));
    float L = 0.0f, O = 0.0f;
    for (int c = 0; c < nchunks; ++c) {
        const float* q = part_ptr<HD>(const_cast<float*>(part), p, kvh, c, g);
        const float l = __ldcg(q + 1);
        if (l > 0.0f) {
            const float w = expf(__ldcg(q) - M);
            L = fmaf(l, w, L);
            O = fmaf(__ldcg(q + 2 + d), w, O);
        }
    }
    return __fdiv_rn(O, L);
}

template <int HD>
__device__ void attn_merge(const AttnDev& p, const float* part, int kvh, int nchunks, float* out, int tid,
                           int nthreads)
{
    for (int e = tid; e < p.gqa * HD; e += nthreads) {
        const int g = e / HD, d = e % HD;
        out[(size_t)(kvh * p.gqa + g) * HD + d] = attn_merge_one<HD>(p, part, kvh, g, d, nchunks);
    }
}

// Merge of every query head's partials into a vector (e.g. the staged input of the O projection):
// out_at(e) receives element e = head * HD + d. Two batched passes over the partials: the
// statistics (m, l) of every (head, chunk) into shared scratch and from them per-chunk weights
// w_c = exp(m_c - M) / L; then o = sum_c o_c[d] w_c. `scratch` holds 2 * heads * nchunks floats.
// attn_merge_heads covers the query heads h0 .. h0 + heads - 1 only (e then counts from h0 * HD).
template <int HD, typename Sync, typename Out>
__device__ void attn_merge_heads(const AttnDev& p, const float* part, int nchunks, int h0, int heads, float* scratch,
                                 int tid, int nthreads, Sync sync, Out out_at)
{
    float* mw = scratch;                     // [heads][nchunks]: m, then the weight
    float* lw = scratch + heads * nchunks;   // [heads][nchunks]: l
    for (int i = tid; i < heads * nchunks; i += nthreads) {
        const int h = h0 + i / nchunks, c = i % nchunks;
        const float* q = part_ptr<HD>(const_cast<float*>(part), p, h / p.gqa, c, h % p.gqa);
        mw[i] = __ldcg(q);
        lw[i] = __ldcg(q + 1);
    }
    sync();
    for (int h = tid; h < heads; h += nthreads) {
        float M = -INFINITY;
        for (int c = 0; c < nchunks; ++c)
            M = fmaxf(M, mw[h * nchunks + c]);
        float L = 0.0f;
        for (int c = 0; c < nchunks; ++c) {
            const float l = lw[h * nchunks + c];
            const float w = l > 0.0f ? expf(mw[h * nchunks + c] - M) : 0.0f;
            mw[h * nchunks + c] = w;
            L = fmaf(l, w, L);
        }
        const float inv = __fdiv_rn(1.0f, L);
        for (int c = 0; c < nchunks; ++c)
            mw[h * nchunks + c] *= inv;
    }
    sync();
    for (int e = tid; e < heads * HD; e += nthreads) {
        const int hl = e / HD, h = h0 + hl, d = e % HD;
        const float* w = mw + hl * nchunks;
        float o = 0.0f;
        int c = 0;
        for (; c + 4 <= nchunks; c += 4) {
            float v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                v[u] = __ldcg(part_ptr<HD>(const_cast<float*>(part), p, h / p.gqa, c + u, h % p.gqa) + 2 + d);
#pragma unroll
            for (int u = 0; u < 4; ++u)
                o = fmaf(v[u], w[c + u], o);
        }
        for (; c < nchunks; ++c)
            o = fmaf(__ldcg(part_ptr<HD>(const_cast<float*>(part), p, h / p.gqa, c, h % p.gqa) + 2 + d), w[c], o);
        out_at(e, o);
    }
}

template <int HD, typename Sync, typename Out>
__device__ void attn_merge_all(const AttnDev& p, const float* part, int nchunks, float* scratch, int tid, int nthreads,
                               Sync sync, Out out_at)
{
    attn_merge_heads<HD>(p, part, nchunks, 0, p.kv_heads * p.gqa, scratch, tid, nthreads, sync, out_at);
}

struct BlockSync {
    __device__ __forceinline__ void operator()() const { __syncthreads(); }
};

// One work item (kvh, chunk) of the attention at position `pos`, run by threads tid in [0, nthreads)
// of a CTA (nthreads a multiple of 32, at least 128). `sm` holds attn_smem_floats(HD, gqa) floats, `cs`
// HD doubles. When `out` is non-null and the item is the only chunk, the normalised output is written
// there; otherwise the partial (m, l, o) goes to `part`.
struct NoWait {
    __device__ void operator()() const {}
};

// `wait` runs after the loads of cache rows written by earlier steps (and of the RoPE table) are
// issued and before q_in is read: a kernel launched early uses it to wait for the kernel that
// produced q_in.
template <typename KV, int HD, bool FUSED, typename Sync, typename Wait = NoWait>
__device__ __forceinline__ void attention_item(const AttnDev& p, const float* q_in, KV* kc, KV* vc, int pos, int kvh, int chunk,
                               float* out, float* part, float* sm, double* cs, int tid, int nthreads, Sync sync,
                               Wait wait = Wait{})
{
    constexpr int LD = HD + 1;
    const int G = p.gqa;
    float* Ks = sm;                   // [kAttnKeys][LD]
    float* Vs = Ks + kAttnKeys * LD;  // [kAttnKeys][LD]
    float* Qs = Vs + kAttnKeys * LD;  // [G][HD]
    float* Ps = Qs + G * HD;          // [G][kAttnKeys]
    float* Ms = Ps + G * kAttnKeys;   // [G]
    float* Ls = Ms + G;               // [G]

    const int n = pos + 1;
    const int nchunks = (n + kAttnKeys - 1) / kAttnKeys;
    const int key0 = chunk * kAttnKeys;
    const int nk = min(kAttnKeys, n - key0);
    const size_t head_base = (size_t)kvh * p.max_seq * HD;
    const bool holds_new = FUSED && (chunk == nchunks - 1);
    const int t_new = holds_new ? pos - key0 : -1;  // tile row of the key appended by this step

    // K/V tile rows written by earlier steps, as 16-byte vectors: the first batch is issued before
    // the RoPE work below so that both sets of loads are in flight together.
    constexpr int VEC = 16 / (int)sizeof(KV);
    constexpr int VPR = HD / VEC;
    constexpr int BATCH = 4;
    const int nvec = nk * VPR;
    uint4 kreg[BATCH], vreg[BATCH];
#define MUYO_KV_LOAD_BATCH(BASE)                                                                      \
    _Pragma("unroll") for (int u = 0; u < BATCH; ++u)                                                 \
    {                                                                                                 \
        const int v = (BASE) + u * nthreads + tid;                                                    \
        const int t = v / VPR;                                                                        \
        if (v < nvec && t != t_new) {                                                                 \
            const size_t off = head_base + (size_t)(key0 + t) * HD + (size_t)(v % VPR) * VEC;         \
            kreg[u] = __ldcg(reinterpret_cast<const uint4*>(kc + off));                              \
            vreg[u] = __ldcg(reinterpret_cast<const uint4*>(vc + off));                              \
        }                                                                                             \
    }
#define MUYO_KV_STORE_BATCH(BASE)                                                                     \
    _Pragma("unroll") for (int u = 0; u < BATCH; ++u)                                                 \
    {                                                                                                 \
        const int v = (BASE) + u * nthreads + tid;                                                    \
        const int t = v / VPR;                                                                        \
        if (v < nvec && t != t_new) {                                                                 \
            const int c0 = (v % VPR) * VEC;                                                           \
            const KV* kk = reinterpret_cast<const KV*>(&kreg[u]);                                     \
            const KV* vv = reinterpret_cast<const KV*>(&vreg[u]);                                     \
            _Pragma("unroll") for (int i = 0; i < VEC; ++i)                                           \
            {                                                                                         \
                Ks[t * LD + c0 + i] = kv_value<KV>(kk[i]);                                            \
                Vs[t * LD + c0 + i] = kv_value<KV>(vv[i]);                                            \
            }                                                                                         \
        }                                                                                             \
    }
    MUYO_KV_LOAD_BATCH(0)
    // cos/sin of frequency j = tid at this position (HD / 2 <= 64 < nthreads): table loads issued now.
    double rc = 0.0, rs = 0.0;
    if (FUSED && tid < HD / 2 && p.rope_cs) {
        rc = __ldg(p.rope_cs + (size_t)pos * HD + tid);
        rs = __ldg(p.rope_cs + (size_t)pos * HD + HD / 2 + tid);
    }
    wait();
    // The projections of this step: rows of q, and the new key and value.
    constexpr int QP = (kAttnMaxGroup * (HD / 2) + 127) / 128;  // q pairs per thread (nthreads >= 128)
    constexpr int VP = (HD + 127) / 128;                        // new-value elements per thread
    float2 qreg[QP];
    float2 knew = make_float2(0.f, 0.f);
    float vnew[VP];
    if (FUSED) {
#pragma unroll
        for (int i = 0; i < QP; ++i) {
            const int e = tid + i * nthreads;
            if (e < G * (HD / 2)) {
                const int g = e / (HD / 2), j = e % (HD / 2);
                const float* qh = q_in + (size_t)(kvh * G + g) * HD;
                qreg[i] = make_float2(__ldcg(qh + j), __ldcg(qh + j + HD / 2));
            }
        }
        if (holds_new) {
            const int qd = p.heads * HD, kvd = p.kv_heads * HD;
            const float* kr = q_in + qd + (size_t)kvh * HD;
            const float* vr = q_in + qd + kvd + (size_t)kvh * HD;
            if (tid < HD / 2)
                knew = make_float2(__ldcg(kr + tid), __ldcg(kr + tid + HD / 2));
#pragma unroll
            for (int i = 0; i < VP; ++i)
                if (tid + i * nthreads < HD)
                    vnew[i] = __ldcg(vr + tid + i * nthreads);
        }
    }

    if (FUSED) {
        if (tid < HD / 2) {
            if (!p.rope_cs)
                rope_cs_f64(pos, tid, HD, p.rope_base, rc, rs);
            cs[tid] = rc;
            cs[HD / 2 + tid] = rs;
        }
        sync();
#pragma unroll
        for (int i = 0; i < QP; ++i) {
            const int e = tid + i * nthreads;
            if (e < G * (HD / 2)) {
                const int g = e / (HD / 2), j = e % (HD / 2);
                float y0, y1;
                rope_pair_f64(qreg[i].x, qreg[i].y, cs[j], cs[HD / 2 + j], y0, y1);
                Qs[g * HD + j] = y0;
                Qs[g * HD + j + HD / 2] = y1;
            }
        }
        if (holds_new) {
            if (tid < HD / 2) {
                const int j = tid;
                float y0, y1;
                rope_pair_f64(knew.x, knew.y, cs[j], cs[HD / 2 + j], y0, y1);
                const KV k0 = kv_round<KV>(y0), k1 = kv_round<KV>(y1);
                kc[head_base + (size_t)pos * HD + j] = k0;
                kc[head_base + (size_t)pos * HD + j + HD / 2] = k1;
                Ks[t_new * LD + j] = kv_value<KV>(k0);
                Ks[t_new * LD + j + HD / 2] = kv_value<KV>(k1);
            }
#pragma unroll
            for (int i = 0; i < VP; ++i) {
                const int d = tid + i * nthreads;
                if (d < HD) {
                    const KV v0 = kv_round<KV>(vnew[i]);
                    vc[head_base + (size_t)pos * HD + d] = v0;
                    Vs[t_new * LD + d] = kv_value<KV>(v0);
                }
            }
        }
    } else {
        for (int e = tid; e < G * HD; e += nthreads)
            Qs[e] = __ldcg(q_in + (size_t)kvh * G * HD + e);
    }
    MUYO_KV_STORE_BATCH(0)
    for (int base = BATCH * nthreads; base < nvec; base += BATCH * nthreads) {
        MUYO_KV_LOAD_BATCH(base)
        MUYO_KV_STORE_BATCH(base)
    }
#undef MUYO_KV_LOAD_BATCH
#undef MUYO_KV_STORE_BATCH
    sync();

    // Scores: thread (t, h0) computes key t for group members g = h0, h0 + hs, ...
    {
        const int t = tid % kAttnKeys, h0 = tid / kAttnKeys, hs = nthreads / kAttnKeys;
        if (h0 < hs) {
            for (int g = h0; g < G; g += hs) {
                float s = -INFINITY;
                if (t < nk) {
                    float dot = 0.0f;
#pragma unroll 16
                    for (int d = 0; d < HD; ++d)
                        dot = fmaf(Qs[g * HD + d], Ks[t * LD + d], dot);
                    s = dot * p.scale;
                }
                Ps[g * kAttnKeys + t] = s;
            }
        }
    }
    sync();
    // Softmax statistics per group member: one warp per member.
    {
        const int lane = tid & 31, warp = tid >> 5, nw = nthreads / 32;
        for (int g = warp; g < G; g += nw) {
            float m = -INFINITY;
            for (int t = lane; t < kAttnKeys; t += 32)
                m = fmaxf(m, Ps[g * kAttnKeys + t]);
            m = warp_max(m);
            float l = 0.0f;
            for (int t = lane; t < kAttnKeys; t += 32) {
                const float s = Ps[g * kAttnKeys + t];
                const float e = t < nk ? expf(s - m) : 0.0f;
                Ps[g * kAttnKeys + t] = e;
                l += e;
            }
            l = warp_sum(l);
            if (lane == 0) {
                Ms[g] = m;
                Ls[g] = l;
            }
        }
    }
    sync();
    // Unnormalised P.V for this chunk.
    const bool single = out != nullptr && nchunks == 1;
    for (int e = tid; e < G * HD; e += nthreads) {
        const int g = e / HD, d = e % HD;
        float o = 0.0f;
        for (int t = 0; t < nk; ++t)
            o = fmaf(Ps[g * kAttnKeys + t], Vs[t * LD + d], o);
        if (single) {
            out[(size_t)(kvh * G + g) * HD + d] = __fdiv_rn(o, Ls[g]);
        } else {
            float* pp = part_ptr<HD>(part, p, kvh, chunk, g);
            pp[2 + d] = o;
            if (d == 0) {
                pp[0] = Ms[g];
                pp[1] = Ls[g];
            }
        }
    }
}

struct PdlWaitTrigger {
    __device__ void operator()() const
    {
        pdl_wait();
        pdl_trigger();
    }
};

// Standalone attention: grid (kv_heads, max_chunks), CTAs past the current chunk count exit. The
// position and the cache rows of earlier steps are read before pdl_wait (they were written two or
// more kernels back); q_in after it.
template <typename KV, int HD, bool FUSED, bool INLINE_MERGE>
__global__ void __launch_bounds__(kAttnThreads) k_attention(AttnDev p, const float* __restrict__ q_in,
                                                             KV* __restrict__ kc, KV* __restrict__ vc,
                                                             const int32_t* __restrict__ pos_ptr,
                                                             float* __restrict__ out, float* __restrict__ part,
                                                             int32_t* __restrict__ counters)
{
    extern __shared__ float sm[];
    __shared__ double cs[HD];
    __shared__ int last_flag;
    const int kvh = blockIdx.x, chunk = blockIdx.y;
    const int pos = pos_ptr ? __ldcg(pos_ptr) : p.n_keys_fixed - 1;
    if (pos < 0 || pos >= p.max_seq)
        return;  // a device position outside the cache: nothing is read or written
    const int nchunks = (pos + 1 + kAttnKeys - 1) / kAttnKeys;
    if (chunk >= nchunks)
        return;
    attention_item<KV, HD, FUSED>(p, q_in, kc, vc, pos, kvh, chunk, out, part, sm, cs, threadIdx.x, blockDim.x,
                                  BlockSync{}, PdlWaitTrigger{});
    if (nchunks == 1 || !INLINE_MERGE)
        return;
    // Last CTA of this KV head merges the chunks, then re-arms the counter for the next launch.
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const int ticket = atomicAdd(&counters[kvh], 1);
        last_flag = ticket == nchunks - 1;
    }
    __syncthreads();
    if (!last_flag)
        return;
    __threadfence();
    if (2 * p.gqa * nchunks <= attn_smem_floats(HD, p.gqa)) {
        // Batched merge in the (now free) item scratch: one pass of statistics, one of values.
        float* o = out + (size_t)kvh * p.gqa * HD;
        attn_merge_heads<HD>(p, part, nchunks, kvh * p.gqa, p.gqa, sm, threadIdx.x, blockDim.x, BlockSync{},
                             [o](int e, float v) { o[e] = v; });
    } else {
        attn_merge<HD>(p, part, kvh, nchunks, out, threadIdx.x, blockDim.x);
    }
    if (threadIdx.x == 0)
        counters[kvh] = 0;
}

template <int HD>
__global__ void __launch_bounds__(kAttnThreads) k_attention_combine(AttnDev p, const int32_t* __restrict__ pos_ptr,
                                                                     const float* __restrict__ part,
                                                                     float* __restrict__ out)
{
    const int kvh = blockIdx.x;
    const int pos = pos_ptr ? __ldcg(pos_ptr) : p.n_keys_fixed - 1;
    if (pos < 0 || pos >= p.max_seq)
        return;
    const int nchunks = (pos + 1 + kAttnKeys - 1) / kAttnKeys;
    if (nchunks <= 1)
        return;  // the single chunk wrote its output directly
    attn_merge<HD>(p, part, kvh, nchunks, out, threadIdx.x, blockDim.x);
}

}  // namespace muyo
