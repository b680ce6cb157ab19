// Split-K GQA decode attention over the persistent KV cache (flash-decoding style).
//
// Grid (kv_heads, chunks): one CTA per (KV head, 64-key chunk). The CTA stages its K and V tiles
// in shared memory once (F16 or F32 cache, converted to F32) and serves all `gqa` query heads of
// the group from them, which is the GQA broadcast of tools/reference_qwen2.py:133 and
// shaders/llama/mul_mat_vec_base.glsl:55-64 without re-reading K/V per query head. Each CTA writes
// (max, sum, unnormalised output) per query head; the chunks are merged either by the last CTA of
// the KV head to finish (a self-resetting arrival counter, used by the fused decode step) or by a
// separate combine kernel (the op-level entry point, whose workspace may hold anything).
//
// With FUSED the CTA also performs the step's KV append: it rotates the raw key with NeoX RoPE in
// double precision (theta = pos * base^(-2j/hd), the rotation of tools/reference_qwen2.py:84-93,
// evaluated in float64 as there and rounded once), rounds key and value to the cache type, and the
// CTA holding the last chunk stores them at row `pos`; that CTA also uses the stored values for
// key `pos` itself, so every CTA reads only rows the previous steps finished writing.
#pragma once

#include "common.cuh"

namespace muyo {

constexpr int kAttnKeys = 64;      // keys per CTA
constexpr int kAttnThreads = 128;  // 4 warps
constexpr int kAttnMaxGroup = 16;  // query heads per KV head

struct AttnDev {
    int heads, kv_heads, gqa, max_seq, n_keys_fixed;
    float scale;
    double rope_base;
    int max_chunks;
};

template <typename KV>
__device__ __forceinline__ float kv_load(const KV* p);
template <>
__device__ __forceinline__ float kv_load<float>(const float* p)
{
    return *p;
}
template <>
__device__ __forceinline__ float kv_load<__half>(const __half* p)
{
    return __half2float(*p);
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

// Shared-memory footprint of the attention CTA (floats).
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

template <int HD>
__device__ void attn_merge(const AttnDev& p, const float* part, int kvh, int nchunks, float* out)
{
    for (int e = threadIdx.x; e < p.gqa * HD; e += blockDim.x) {
        const int g = e / HD, d = e % HD;
        float M = -INFINITY;
        for (int c = 0; c < nchunks; ++c)
            M = fmaxf(M, part_ptr<HD>(const_cast<float*>(part), p, kvh, c, g)[0]);
        float L = 0.0f, O = 0.0f;
        for (int c = 0; c < nchunks; ++c) {
            const float* q = part_ptr<HD>(const_cast<float*>(part), p, kvh, c, g);
            if (q[1] > 0.0f) {
                const float w = expf(q[0] - M);
                L = fmaf(q[1], w, L);
                O = fmaf(q[2 + d], w, O);
            }
        }
        out[(size_t)(kvh * p.gqa + g) * HD + d] = __fdiv_rn(O, L);
    }
}

// q_in: FUSED -> raw projections [heads*hd | kv_heads*hd (k) | kv_heads*hd (v)]; else rotated q.
template <typename KV, int HD, bool FUSED, bool INLINE_MERGE>
__global__ void __launch_bounds__(kAttnThreads) k_attention(AttnDev p, const float* __restrict__ q_in,
                                                             KV* __restrict__ kc, KV* __restrict__ vc,
                                                             const int32_t* __restrict__ pos_ptr,
                                                             float* __restrict__ out, float* __restrict__ part,
                                                             int32_t* __restrict__ counters)
{
    extern __shared__ float sm[];
    constexpr int LD = HD + 1;
    const int G = p.gqa;
    float* Ks = sm;                          // [kAttnKeys][LD]
    float* Vs = Ks + kAttnKeys * LD;         // [kAttnKeys][LD]
    float* Qs = Vs + kAttnKeys * LD;         // [G][HD]
    float* Ps = Qs + G * HD;                 // [G][kAttnKeys]
    float* Ms = Ps + G * kAttnKeys;          // [G]
    float* Ls = Ms + G;                      // [G]
    float* Kn = Ls + G;                      // [HD] new key (rounded)
    float* Vn = Kn + HD;                     // [HD] new value (rounded)
    __shared__ double cs[HD];                // cos at [j], sin at [HD/2 + j]
    __shared__ int last_flag;

    const int kvh = blockIdx.x, chunk = blockIdx.y;
    const int pos = pos_ptr ? *pos_ptr : p.n_keys_fixed - 1;
    if (pos < 0 || pos >= p.max_seq)
        return;  // a device position outside the cache: nothing is read or written
    const int n = pos + 1;
    const int nchunks = (n + kAttnKeys - 1) / kAttnKeys;
    if (chunk >= nchunks)
        return;
    const int key0 = chunk * kAttnKeys;
    const int nk = min(kAttnKeys, n - key0);
    const size_t head_base = (size_t)kvh * p.max_seq * HD;
    const bool holds_new = FUSED && (chunk == nchunks - 1);

    if (FUSED) {
        if (threadIdx.x < HD / 2) {
            double c, s;
            rope_cs_f64(pos, threadIdx.x, HD, p.rope_base, c, s);
            cs[threadIdx.x] = c;
            cs[HD / 2 + threadIdx.x] = s;
        }
        __syncthreads();
        const int qd = p.heads * HD, kvd = p.kv_heads * HD;
        for (int e = threadIdx.x; e < G * (HD / 2); e += blockDim.x) {
            const int g = e / (HD / 2), j = e % (HD / 2);
            const float* qh = q_in + (size_t)(kvh * G + g) * HD;
            float y0, y1;
            rope_pair_f64(qh[j], qh[j + HD / 2], cs[j], cs[HD / 2 + j], y0, y1);
            Qs[g * HD + j] = y0;
            Qs[g * HD + j + HD / 2] = y1;
        }
        if (holds_new) {
            const float* kr = q_in + qd + (size_t)kvh * HD;
            const float* vr = q_in + qd + kvd + (size_t)kvh * HD;
            for (int j = threadIdx.x; j < HD / 2; j += blockDim.x) {
                float y0, y1;
                rope_pair_f64(kr[j], kr[j + HD / 2], cs[j], cs[HD / 2 + j], y0, y1);
                const KV k0 = kv_round<KV>(y0), k1 = kv_round<KV>(y1);
                kc[head_base + (size_t)pos * HD + j] = k0;
                kc[head_base + (size_t)pos * HD + j + HD / 2] = k1;
                Kn[j] = kv_load<KV>(&k0);
                Kn[j + HD / 2] = kv_load<KV>(&k1);
            }
            for (int d = threadIdx.x; d < HD; d += blockDim.x) {
                const KV v0 = kv_round<KV>(vr[d]);
                vc[head_base + (size_t)pos * HD + d] = v0;
                Vn[d] = kv_load<KV>(&v0);
            }
        }
    } else {
        for (int e = threadIdx.x; e < G * HD; e += blockDim.x)
            Qs[e] = q_in[(size_t)kvh * G * HD + e];
    }
    __syncthreads();  // Kn / Vn are read by other threads below

    // Stage the K and V tiles (keys that earlier steps wrote; the new key comes from Kn/Vn).
    for (int e = threadIdx.x; e < kAttnKeys * HD; e += blockDim.x) {
        const int t = e / HD, d = e % HD;
        const int j = key0 + t;
        float kv = 0.0f, vv = 0.0f;
        if (t < nk) {
            if (holds_new && j == pos) {
                kv = Kn[d];
                vv = Vn[d];
            } else {
                kv = kv_load<KV>(kc + head_base + (size_t)j * HD + d);
                vv = kv_load<KV>(vc + head_base + (size_t)j * HD + d);
            }
        }
        Ks[t * LD + d] = kv;
        Vs[t * LD + d] = vv;
    }
    __syncthreads();

    // Scores: thread (t, half) computes keys t for group members g = half, half + 2, ...
    {
        const int t = threadIdx.x % kAttnKeys, h0 = threadIdx.x / kAttnKeys, hs = kAttnThreads / kAttnKeys;
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
    __syncthreads();
    // Softmax statistics per group member: one warp per member.
    {
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = kAttnThreads / 32;
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
    __syncthreads();
    // Unnormalised P.V for this chunk.
    const bool single = nchunks == 1;
    for (int e = threadIdx.x; e < G * HD; e += blockDim.x) {
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
    if (single || !INLINE_MERGE)
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
    attn_merge<HD>(p, part, kvh, nchunks, out);
    if (threadIdx.x == 0)
        counters[kvh] = 0;
}

template <int HD>
__global__ void __launch_bounds__(kAttnThreads) k_attention_combine(AttnDev p, const int32_t* __restrict__ pos_ptr,
                                                                     const float* __restrict__ part,
                                                                     float* __restrict__ out)
{
    const int kvh = blockIdx.x;
    const int pos = pos_ptr ? *pos_ptr : p.n_keys_fixed - 1;
    if (pos < 0 || pos >= p.max_seq)
        return;
    const int nchunks = (pos + 1 + kAttnKeys - 1) / kAttnKeys;
    if (nchunks <= 1)
        return;  // the single chunk wrote its output directly
    attn_merge<HD>(p, part, kvh, nchunks, out);
}

}  // namespace muyo
