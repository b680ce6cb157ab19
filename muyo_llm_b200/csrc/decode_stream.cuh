// The streaming decode kernel: every decode step of a generate call in ONE cooperative launch, one
// CTA per SM (the persistent engine, engine 0).
//
// A batch-1 Qwen2 step is a chain of ~5 dependent phases per layer (QKV, attention, O, gate/up,
// down) plus the LM head, each moving 0.3-17 MB of weights. Two costs dominate when the phases run
// as separate kernels: the weights of a phase cannot start streaming before the phase's kernel is
// resident, and every hand-off between phases is a grid-wide completion plus a reload of the input.
// This kernel removes both:
//
//   weights    warp 8 of every CTA (the producer) walks the static schedule of the weight rows its SM
//              consumes in the whole call (layer by layer, phase by phase, then the LM head, step
//              after step) and bulk-copies them (cp.async.bulk) into a byte-granular ring of shared
//              memory, one piece of whole rows at a time, each piece guarded by a full/empty mbarrier
//              pair. The ring holds most of a layer, so the weights of later phases arrive while the
//              current phase waits on its inputs. The producer keeps only a few pieces in flight
//              while a layer runs (28 KB pieces, 2 deep: deep copy queues stretch the latency of the
//              activation hand-offs) and more for the LM head (28 KB, 6 deep), which has no chain.
//   hand-offs  every activation a phase produces (q/k/v, attention partials, h1, the SwiGLU output,
//              the layer output) is written as 64-bit words {tag, value}: a single-copy-atomic store
//              whose upper half is the step's tag. A consumer polls the words it needs until every
//              tag matches: the data and its readiness arrive in one L2 round trip, with no barrier,
//              counter or fence. Each layer has its own buffers and every CTA publishes its greedy
//              candidate every step, so within a step each word is written once, and the next step's
//              writes wait (through the data they depend on) for every CTA to finish reading.
//   greedy     each CTA publishes its best (logit, index) of its LM-head rows and reads every CTA's
//              pair, so every CTA derives the same next token without a grid barrier (a fence on
//              each side orders the step's KV-cache rows before the next step reads them).
//
// Per layer, CTA c owns a contiguous row range of every matrix (rows split evenly over the grid);
// warps take the rows of a piece (the K range split over warps when a piece has fewer than 8 rows),
// lanes the 16-byte chunks of a row in shared memory, x staged in shared memory in the split layout
// of gemv.cuh. Attention work items are (query head, key range) pairs: 64-key sub-tiles with an
// online softmax, K and V of the next sub-tile loaded into registers while the current one computes;
// the O phase merges the items' (max, sum, output) partials while staging its input.
//
// Every wait (mbarrier, tagged word) is bounded by the global timer: on expiry the CTA sets the
// launch's abort word and the model's error word, and every wait of every CTA then gives up at once;
// the producer drains its copies before the CTA exits.
#pragma once

#include "attention.cuh"
#include "common.cuh"
#include "gemv.cuh"
#include "sync.cuh"

namespace muyo {

typedef unsigned long long u64;

constexpr int kSWarps = 7;                   // consumer warps (+ the producer: 2 warps per scheduler)
constexpr int kSCThreads = kSWarps * 32;     // consumer threads
constexpr int kSThreads = kSCThreads + 32;   // + the producer warp
constexpr int kSAttnThreads = 128;           // threads of an attention item's arithmetic
constexpr int kSBars = 32;                   // piece barrier slots (pieces outstanding at most)
constexpr int kSJmax = 4;                    // key ranges per query head
constexpr int kSKeys = 64;                   // keys per attention sub-tile
constexpr unsigned kSLayerPiece = 28672;     // target bytes of a layer weight piece
constexpr unsigned kSHeadPiece = 28672;      // target bytes of an LM-head piece
constexpr int kSLayerDepth = 2;              // pieces in flight while a layer runs
constexpr int kSHeadDepth = 6;               // pieces in flight while the LM head runs
constexpr int kSErrTimeout = 3;              // the model's error word on an expired wait

enum SPhase { SP_QKV = 0, SP_O = 1, SP_GU = 2, SP_DOWN = 3, SP_HEAD = 4 };

struct SLayer {
    const __half* wqkv;
    const float* bqkv;
    const float* attn_norm;
    const __half* wo;
    const float* ffn_norm;
    const __half* wgate;
    const __half* wup;
    const __half* wdown;
};

struct SArgs {
    const SLayer* layers;
    int L, H, F, V, QKV, QD, KVD, heads, kv_heads, gqa, max_seq;
    float eps, scale;
    const __half* embd;
    const __half* lm;
    const float* final_norm;
    const double* rope_cs;  // [max_seq][hd]: cos theta_j at [pos*hd + j], sin at [pos*hd + hd/2 + j]
    void* kc;
    void* vc;
    long long kv_layer_elems;
    u64* ll;                // tagged words: one block per layer
    long long ll_layer;     // words per layer block
    int o_qkv, o_part, o_h1, o_act, o_hout;  // word offsets inside a block
    u64* ll_best;           // [2][grid][2]: per CTA {value, index} words, double-buffered by step
    float* logits;
    Control* ctrl;
    int32_t* tokens;
    int* err;               // the model's error word
    int* abort_g;           // this launch's abort word (zeroed before the launch)
    unsigned tag0;          // tag of the first step (never 0: the buffers start zeroed)
    int pos0, prompt_end, total, n_steps;
    int ring_bytes;         // R, a multiple of 128
    int off_work, off_hraw, off_h1raw, off_misc;  // byte offsets in dynamic shared memory
    int xs_floats;          // floats of the staged input (max(H, QD, F))
};

// ---- small helpers ------------------------------------------------------------------------------------

__device__ __forceinline__ void s_bar() { asm volatile("bar.sync 1, %0;" ::"r"(kSCThreads) : "memory"); }

__device__ __forceinline__ void ll_put(u64* p, unsigned bits, unsigned tag)
{
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(((u64)tag << 32) | bits) : "memory");
}
__device__ __forceinline__ void ll_putf(u64* p, float v, unsigned tag) { ll_put(p, __float_as_uint(v), tag); }

__device__ __forceinline__ u64 ll_get(const u64* p)
{
    u64 v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void ll_get2(const u64* p, u64& a, u64& b)
{
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ unsigned ll_tag(u64 w) { return (unsigned)(w >> 32); }
__device__ __forceinline__ float ll_val(u64 w) { return __uint_as_float((unsigned)w); }

__device__ __forceinline__ bool s_aborted(const SArgs& a) { return *reinterpret_cast<volatile int*>(a.abort_g) != 0; }

__device__ __forceinline__ void s_fail(const SArgs& a)
{
    atomicExch(a.abort_g, 1);
    atomicMax(a.err, kSErrTimeout);
}

// Bounded wait for the phase of `b` with the given parity. False when the launch aborted or the wait
// expired (which aborts it). A failed test sleeps briefly: a warp spinning on shared memory never
// stalls, and the scheduler would otherwise keep issuing it ahead of the warps doing the work.
__device__ __forceinline__ bool s_wait(const SArgs& a, uint64_t* b, unsigned parity)
{
    if (mbar_try_wait(b, parity))
        return true;
    const unsigned long long t0 = now_ns();
    for (int k = 1;; ++k) {
        __nanosleep(20);
        if (mbar_try_wait(b, parity))
            return true;
        if ((k & 15) == 0) {
            if (s_aborted(a))
                return false;
            if (now_ns() - t0 > kWaitLimitNs) {
                s_fail(a);
                return false;
            }
        }
    }
}

// Shared-memory regions of a CTA (byte offsets in SArgs).
struct SSmem {
    char* ring;
    float* xs;      // staged input vector, split layout (xs_floats; the first hidden floats for QKV, GU)
    float* stats;   // merge: the staged partials [heads][J][hd + 2], then the weights [heads][J]
    float* attn;    // attention scratch
    float* hraw;    // the layer input (the O projection's residual)
    float* h1raw;   // h1 (the down projection's residual)
    uint64_t* full;
    uint64_t* empty;
    u64* pstart;    // producer: virtual start offset of each outstanding piece
    float* red;     // [32]
    float* psum;    // [2][2][64] K-split partial sums
    float* bestv;   // [kSWarps]
    int* besti;     // [kSWarps]
    int* greedy;    // [1]
};

// Misc region: barriers first (8-byte aligned).
__host__ __device__ constexpr int s_misc_bytes()
{
    return 2 * kSBars * 8 + kSBars * 8 + 32 * 4 + 2 * 2 * 64 * 4 + kSWarps * 4 + kSWarps * 4 + 16;
}

__device__ __forceinline__ SSmem s_smem(const SArgs& a, char* base, int heads)
{
    SSmem s;
    s.ring = base;
    s.xs = reinterpret_cast<float*>(base + a.off_work);
    // After the O projection's input (q_dim == hidden floats): the merge's staged partials, or (earlier
    // in the same phase sequence of a CTA) the attention scratch.
    s.stats = s.xs + (a.QD + 3) / 4 * 4;
    s.attn = s.stats;
    s.hraw = reinterpret_cast<float*>(base + a.off_hraw);
    s.h1raw = reinterpret_cast<float*>(base + a.off_h1raw);
    char* m = base + a.off_misc;
    s.full = reinterpret_cast<uint64_t*>(m);
    s.empty = s.full + kSBars;
    s.pstart = reinterpret_cast<u64*>(s.empty + kSBars);
    s.red = reinterpret_cast<float*>(s.pstart + kSBars);
    s.psum = s.red + 32;
    s.bestv = s.psum + 2 * 2 * 64;
    s.besti = reinterpret_cast<int*>(s.bestv + kSWarps);
    s.greedy = s.besti + kSWarps;
    return s;
}

// ---- the weight schedule (shared by the producer and the consumers) -----------------------------------

struct SGeom {
    const __half* w0;
    const __half* w1;
    int K, nmat, rb, re, rpp;
};

// Rows of a piece: as many whole rows (of every matrix of the phase) as fit the target size, at least
// one, in multiples of the consumer warps where there are enough (one row, or two for the LM head, per
// warp).
__host__ __device__ inline int s_rows_per_piece(int K, int nmat, bool head)
{
    const unsigned rowset = (unsigned)K * 2u * (unsigned)nmat;
    int n = (int)((head ? kSHeadPiece : kSLayerPiece) / rowset);
    if (n < 1)
        n = 1;
    if (n >= kSWarps)
        n = n / kSWarps * kSWarps;
    return n;
}

__device__ __forceinline__ SGeom s_geom(const SArgs& a, int l, int ph)
{
    SGeom g;
    int M;
    g.w1 = nullptr;
    g.nmat = 1;
    if (ph == SP_HEAD) {
        g.w0 = a.lm;
        M = a.V;
        g.K = a.H;
    } else {
        const SLayer& L = a.layers[l];
        switch (ph) {
            case SP_QKV: g.w0 = L.wqkv; M = a.QKV; g.K = a.H; break;
            case SP_O: g.w0 = L.wo; M = a.H; g.K = a.QD; break;
            case SP_GU: g.w0 = L.wgate; g.w1 = L.wup; g.nmat = 2; M = a.F; g.K = a.H; break;
            default: g.w0 = L.wdown; M = a.H; g.K = a.F; break;
        }
    }
    g.rb = (int)((long long)M * blockIdx.x / gridDim.x);
    g.re = (int)((long long)M * (blockIdx.x + 1) / gridDim.x);
    g.rpp = s_rows_per_piece(g.K, g.nmat, ph == SP_HEAD);
    return g;
}

// Position of the producer or a consumer in the ring: the virtual byte offset (bytes placed so far,
// with the skips at the ring's end) and the same offset within the ring.
struct SRing {
    u64 v;
    unsigned p;
};

// Place a piece of `placed` bytes in the ring (never across its end): returns its virtual start, sets
// `phys` to its offset in the ring, and advances the position.
__device__ __forceinline__ u64 s_place(SRing& r, unsigned placed, unsigned R, unsigned& phys)
{
    if (r.p + placed > R) {
        r.v += R - r.p;
        r.p = 0;
    }
    const u64 start = r.v;
    phys = r.p;
    r.v += placed;
    r.p += placed;
    if (r.p == R)
        r.p = 0;
    return start;
}

__device__ __forceinline__ unsigned s_round128(unsigned b) { return (b + 127u) & ~127u; }

// ---- producer -------------------------------------------------------------------------------------------

__device__ __forceinline__ void s_producer(const SArgs& a)
{
    extern __shared__ __align__(128) char smem[];
    const SSmem S = s_smem(a, smem, a.heads);
    const unsigned R = (unsigned)a.ring_bytes;
    SRing pos{0, 0};
    u64 idx = 0, tail = 0;
    bool ok = true;
    for (int step = 0; step < a.n_steps && ok; ++step) {
        for (int l = 0; l <= a.L && ok; ++l) {
            const int nph = l < a.L ? 4 : 1;
            for (int q = 0; q < nph && ok; ++q) {
                const int ph = l < a.L ? q : SP_HEAD;
                const SGeom g = s_geom(a, l, ph);
                const u64 depth = ph == SP_HEAD ? kSHeadDepth : kSLayerDepth;
                for (int r0 = g.rb; r0 < g.re && ok; r0 += g.rpp) {
                    const int n = min(g.rpp, g.re - r0);
                    const unsigned part = (unsigned)n * (unsigned)g.K * 2u;
                    unsigned phys;
                    const u64 start = s_place(pos, s_round128(part * g.nmat), R, phys);
                    const u64 t = idx++;
                    // Ring space: every piece starting before pos.v - R must have been consumed, and at
                    // most kSBars pieces may be outstanding (one barrier pair each).
                    while (ok && tail < t && (S.pstart[tail % kSBars] + R < pos.v || t - tail >= (u64)kSBars)) {
                        ok = s_wait(a, &S.empty[tail % kSBars], (unsigned)((tail / kSBars) & 1));
                        if (ok)
                            ++tail;
                    }
                    // Copies in flight: wait for piece t - depth to land.
                    if (ok && t >= depth)
                        ok = s_wait(a, &S.full[(t - depth) % kSBars], (unsigned)(((t - depth) / kSBars) & 1));
                    if (!ok)
                        break;
                    S.pstart[t % kSBars] = start;
                    char* dst = S.ring + phys;
                    uint64_t* fb = &S.full[t % kSBars];
                    mbar_expect_tx(fb, part * g.nmat);
                    bulk_g2s(dst, g.w0 + (size_t)r0 * g.K, part, fb);
                    if (g.nmat == 2)
                        bulk_g2s(dst + part, g.w1 + (size_t)r0 * g.K, part, fb);
                }
            }
        }
    }
    // Drain: a piece the consumers have released has landed; the others (at most kSBars) are waited
    // for here, so that no copy into this CTA's shared memory is in flight when it exits.
    for (u64 k = tail; k < idx; ++k) {
        const unsigned long long t0 = now_ns();
        while (!mbar_try_wait(&S.full[k % kSBars], (unsigned)((k / kSBars) & 1)) && now_ns() - t0 < kWaitLimitNs)
            __nanosleep(20);
    }
}

// ---- consumers: staging ----------------------------------------------------------------------------------

// Polls words [0, n) of src (n even) until each carries `tag`; this thread handles the pairs
// q = ctid + j * kSCThreads and calls f(q, v0, v1) for each. On abort the remaining pairs are given as 0.
template <typename Fn>
__device__ __forceinline__ void s_poll(const SArgs& a, const u64* src, int n, unsigned tag, int ctid, Fn f)
{
    constexpr int B = 4;
    const int np = n / 2;
    for (int base = 0; base < np; base += B * kSCThreads) {
        u64 x[B][2];
        unsigned pend = 0;
#pragma unroll
        for (int j = 0; j < B; ++j)
            if (base + ctid + j * kSCThreads < np)
                pend |= 1u << j;
        unsigned long long t0 = 0;
        for (int it = 1; pend; ++it) {
#pragma unroll
            for (int j = 0; j < B; ++j)
                if (pend & (1u << j))
                    ll_get2(src + 2 * (base + ctid + j * kSCThreads), x[j][0], x[j][1]);
#pragma unroll
            for (int j = 0; j < B; ++j)
                if ((pend & (1u << j)) && ll_tag(x[j][0]) == tag && ll_tag(x[j][1]) == tag) {
                    f(base + ctid + j * kSCThreads, ll_val(x[j][0]), ll_val(x[j][1]));
                    pend &= ~(1u << j);
                }
            if (pend && (it & 7) == 0) {
                bool give_up = s_aborted(a);
                if (!give_up) {
                    if (t0 == 0) {
                        t0 = now_ns();
                    } else if (now_ns() - t0 > kWaitLimitNs) {
                        s_fail(a);
                        give_up = true;
                    }
                }
                if (give_up) {
#pragma unroll
                    for (int j = 0; j < B; ++j)
                        if (pend & (1u << j))
                            f(base + ctid + j * kSCThreads, 0.0f, 0.0f);
                    pend = 0;
                }
            }
        }
    }
}

// x (natural layout, floats in `x`, this thread's pairs written by itself) -> xs = x / s * w with
// s = sqrt(mean(x^2) + eps) (tools/reference_qwen2.py:81-82), in the split layout. The sum of squares:
// per-thread FMA partials over the thread's pairs, a shuffle tree, the warps' sums in order.
__device__ __forceinline__ void s_norm(const float* x, const float* w, float eps, int K, float* xs, float* red,
                                       int ctid)
{
    const int K8 = K / 8, np = K / 2;
    float ss = 0.0f;
    for (int q = ctid; q < np; q += kSCThreads) {
        const float2 v = reinterpret_cast<const float2*>(x)[q];
        ss = fmaf(v.x, v.x, ss);
        ss = fmaf(v.y, v.y, ss);
    }
    ss = warp_sum(ss);
    if ((ctid & 31) == 0)
        red[ctid >> 5] = ss;
    s_bar();
    float t = 0.0f;
#pragma unroll
    for (int i = 0; i < kSWarps; ++i)
        t += red[i];
    const float s = __fsqrt_rn(__fdiv_rn(t, (float)K) + eps);
    for (int q = ctid; q < np; q += kSCThreads) {
        const float2 v = reinterpret_cast<const float2*>(x)[q];
        const float2 wv = __ldg(reinterpret_cast<const float2*>(w) + q);
        *reinterpret_cast<float2*>(xs + xs_index(2 * q, K8)) = make_float2(__fdiv_rn(v.x, s) * wv.x, __fdiv_rn(v.y, s) * wv.y);
    }
    s_bar();
}

// Merged attention output (the O projection's input, K = heads * HD) from the key-range partials
// (m, l, o) of every (head, range), which sit as heads * J items of HD + 2 tagged words: polled as one
// array into shared memory, then per head M = max_j m_j, w_j = exp(m_j - M) / L with
// L = sum_j l_j exp(m_j - M), and x[h * HD + d] = sum_j o_j[d] w_j (the arithmetic of the step
// graph's merge).
template <int HD>
__device__ __forceinline__ void s_merge(const SArgs& a, const u64* part, int J, unsigned tag, int ctid)
{
    extern __shared__ __align__(128) char smem[];
    const SSmem S = s_smem(a, smem, a.heads);
    constexpr int W = HD + 2;
    const int heads = a.heads, K = a.QD, K8 = K / 8;
    float* stage = S.stats;  // [heads][J][W]
    s_poll(a, part, heads * J * W, tag, ctid,
           [&](int q, float v0, float v1) { reinterpret_cast<float2*>(stage)[q] = make_float2(v0, v1); });
    s_bar();  // every partial staged; every warp is past the previous phase's reads of xs
    float* wgt = stage + heads * J * W;  // [heads][J]
    for (int h = ctid; h < heads; h += kSCThreads) {
        const float* it = stage + (size_t)h * J * W;
        float M = -INFINITY;
        for (int j = 0; j < J; ++j)
            M = fmaxf(M, it[j * W]);
        float L = 0.0f;
        for (int j = 0; j < J; ++j) {
            const float l = it[j * W + 1];
            const float w = l > 0.0f ? expf(it[j * W] - M) : 0.0f;
            wgt[h * J + j] = w;
            L = fmaf(l, w, L);
        }
        const float inv = __fdiv_rn(1.0f, L);
        for (int j = 0; j < J; ++j)
            wgt[h * J + j] *= inv;
    }
    s_bar();
    for (int e = ctid; e < K; e += kSCThreads) {
        const int h = e / HD, d = e % HD;
        const float* it = stage + (size_t)h * J * W + 2 + d;
        float o = 0.0f;
        for (int j = 0; j < J; ++j)
            o = fmaf(it[j * W], wgt[h * J + j], o);
        S.xs[xs_index(e, K8)] = o;
    }
    s_bar();
}

// ---- consumers: attention -------------------------------------------------------------------------------

// Register image of B bytes (a multiple of 4) of cache row data.
template <int B>
struct SRow {
    static constexpr int N = B / 4;
    uint32_t w[N];
};

template <int B>
__device__ __forceinline__ void s_row_load(SRow<B>& r, const void* p)
{
    if constexpr (B % 16 == 0) {
#pragma unroll
        for (int i = 0; i < B / 16; ++i) {
            const uint4 u = __ldcg(reinterpret_cast<const uint4*>(p) + i);
            r.w[4 * i] = u.x;
            r.w[4 * i + 1] = u.y;
            r.w[4 * i + 2] = u.z;
            r.w[4 * i + 3] = u.w;
        }
    } else if constexpr (B % 8 == 0) {
#pragma unroll
        for (int i = 0; i < B / 8; ++i) {
            const uint2 u = __ldcg(reinterpret_cast<const uint2*>(p) + i);
            r.w[2 * i] = u.x;
            r.w[2 * i + 1] = u.y;
        }
    } else {
#pragma unroll
        for (int i = 0; i < SRow<B>::N; ++i)
            r.w[i] = __ldcg(reinterpret_cast<const unsigned*>(p) + i);
    }
}

template <int B>
__device__ __forceinline__ void s_row_zero(SRow<B>& r)
{
#pragma unroll
    for (int i = 0; i < SRow<B>::N; ++i)
        r.w[i] = 0u;
}

// Element i (a compile-time index after unrolling) of a row image of KV values.
template <typename KV, int B>
__device__ __forceinline__ float s_row_elem(const SRow<B>& r, int i)
{
    if constexpr (sizeof(KV) == 2) {
        __half2 h;
        *reinterpret_cast<uint32_t*>(&h) = r.w[i >> 1];
        return (i & 1) ? __high2float(h) : __low2float(h);
    } else {
        return __uint_as_float(r.w[i]);
    }
}

// One layer's attention items handled by this CTA: items (query head h, key range j) for j < J; the
// keys 0..pos are split into 64-key sub-tiles, range j takes sub-tiles [nsub j / J, nsub (j+1) / J).
// Writes each item's (m, l, o[HD]) as tagged words; the range holding key `pos` also rotates the
// step's key with NeoX RoPE (float64 angles and arithmetic, tools/reference_qwen2.py:84-93), rounds
// key and value to the cache type and, for the first head of the KV group, appends them at row pos.
template <typename KV, int HD>
__device__ __forceinline__ void s_attention(const SArgs& a, int l, int pos, int J, unsigned tag, int ctid)
{
    extern __shared__ __align__(128) char smem[];
    const SSmem S = s_smem(a, smem, a.heads);
    constexpr int KQ = HD / 2;                 // K: 2 threads per key, KQ dims each
    constexpr int KB = KQ * (int)sizeof(KV);
    constexpr int VT = HD / 2;                 // V: threads per key row, 2 dims each
    constexpr int VG = kSAttnThreads / VT;     // key groups
    constexpr int VK = kSKeys / VG;            // keys per thread
    constexpr int VB = 2 * (int)sizeof(KV);
    // Loading the next sub-tile's rows while the current one computes would need a second register
    // image; it is off: the kernel is inlined into one body that must not spill (local memory misses
    // the small L1 left beside 227 KB of shared memory).
    constexpr bool PF = false;
    static_assert(VG * VT == kSAttnThreads && VK * VG == kSKeys && 2 * kSKeys == kSAttnThreads && KB % 8 == 0,
                  "attention thread layout");
    double* cs = reinterpret_cast<double*>(S.attn);  // [HD]: cos, then sin
    float* Qs = S.attn + 2 * HD;
    float* Kn = Qs + HD;
    float* Vn = Kn + HD;
    float* Ss = Vn + HD;      // [64]
    float* Ps = Ss + kSKeys;  // [64]
    float* st = Ps + kSKeys;  // [4]: alpha
    float* opart = st + 4;    // [VG][HD]

    const u64* blk = a.ll + (size_t)l * a.ll_layer;
    const u64* qkv = blk + a.o_qkv;
    u64* part = const_cast<u64*>(blk) + a.o_part;
    KV* kc = static_cast<KV*>(a.kc) + (size_t)a.kv_layer_elems * l;
    KV* vc = static_cast<KV*>(a.vc) + (size_t)a.kv_layer_elems * l;
    const int n = pos + 1, nsub = (n + kSKeys - 1) / kSKeys, items = a.heads * J;
    const int warp = ctid >> 5, lane = ctid & 31;
    const bool at = ctid < kSAttnThreads;             // a thread of the item's arithmetic
    const int kt = ctid >> 1, kq = ctid & 1;          // K layout
    const int vd = ctid % VT, vg = ctid / VT;         // V layout

    for (int it = blockIdx.x; it < items; it += gridDim.x) {
        const int h = it / J, j = it % J, g = h / a.gqa;
        const int s0 = nsub * j / J, s1 = nsub * (j + 1) / J;
        const bool has_new = s1 == nsub;
        const size_t hb = (size_t)g * a.max_seq * HD;
        SRow<KB> kr, kn;
        SRow<VB> vr[VK], vn[VK];
        auto load_sub = [&](int s, SRow<KB>& kd, SRow<VB> (&vdst)[VK]) {
            const int key0 = s * kSKeys;
            const int row = key0 + kt;
            if (at && row < n && row != pos)
                s_row_load<KB>(kd, kc + hb + (size_t)row * HD + kq * KQ);
            else
                s_row_zero<KB>(kd);
#pragma unroll
            for (int i = 0; i < VK; ++i) {
                const int r = key0 + vg + VG * i;
                if (at && r < n && r != pos)
                    s_row_load<VB>(vdst[i], vc + hb + (size_t)r * HD + 2 * vd);
                else
                    s_row_zero<VB>(vdst[i]);
            }
        };
        load_sub(s0, kr, vr);  // cache rows of earlier steps: in flight while q is awaited
        double rc = 0.0, rs = 0.0;
        if (ctid < HD / 2) {
            rc = __ldg(a.rope_cs + (size_t)pos * HD + ctid);
            rs = __ldg(a.rope_cs + (size_t)pos * HD + HD / 2 + ctid);
        }
        // q of head h, and (range holding key pos) the step's k and v of group g: one pair per thread.
        {
            const int np = (has_new ? 3 : 1) * (HD / 2);
            const int q = ctid;
            if (q < np) {
                const int which = q / (HD / 2), p2 = 2 * (q % (HD / 2));
                const u64* src = which == 0 ? qkv + (size_t)h * HD + p2
                                 : which == 1 ? qkv + a.QD + (size_t)g * HD + p2
                                              : qkv + a.QD + a.KVD + (size_t)g * HD + p2;
                float* dst = which == 0 ? Qs + p2 : which == 1 ? Kn + p2 : Vn + p2;
                u64 w0, w1;
                unsigned long long t0 = 0;
                for (int k = 1;; ++k) {
                    ll_get2(src, w0, w1);
                    if (ll_tag(w0) == tag && ll_tag(w1) == tag)
                        break;
                    if ((k & 7) == 0) {
                        if (s_aborted(a))
                            break;
                        if (t0 == 0)
                            t0 = now_ns();
                        else if (now_ns() - t0 > kWaitLimitNs) {
                            s_fail(a);
                            break;
                        }
                    }
                }
                dst[0] = ll_val(w0);
                dst[1] = ll_val(w1);
            }
            if (ctid < HD / 2) {
                cs[ctid] = rc;
                cs[HD / 2 + ctid] = rs;
            }
        }
        s_bar();
        // RoPE (q by threads < HD/2, k by HD/2 .. HD-1), rounding of k and v to the cache type, append.
        const bool append = has_new && h % a.gqa == 0;
        if (ctid < HD / 2) {
            float y0, y1;
            rope_pair_f64(Qs[ctid], Qs[ctid + HD / 2], cs[ctid], cs[HD / 2 + ctid], y0, y1);
            Qs[ctid] = y0;
            Qs[ctid + HD / 2] = y1;
        } else if (has_new && ctid < HD) {
            const int jj = ctid - HD / 2;
            float y0, y1;
            rope_pair_f64(Kn[jj], Kn[jj + HD / 2], cs[jj], cs[HD / 2 + jj], y0, y1);
            const KV k0 = kv_round<KV>(y0), k1 = kv_round<KV>(y1);
            Kn[jj] = kv_value<KV>(k0);
            Kn[jj + HD / 2] = kv_value<KV>(k1);
            if (append) {
                kc[hb + (size_t)pos * HD + jj] = k0;
                kc[hb + (size_t)pos * HD + jj + HD / 2] = k1;
                __threadfence();
            }
        }
        if (has_new)
            for (int d = ctid; d < HD; d += kSCThreads) {
                const KV v0 = kv_round<KV>(Vn[d]);
                Vn[d] = kv_value<KV>(v0);
                if (append) {
                    vc[hb + (size_t)pos * HD + d] = v0;
                    __threadfence();
                }
            }
        s_bar();

        float m_run = -INFINITY, l_run = 0.0f, o_run = 0.0f;
        for (int s = s0; s < s1; ++s) {
            if (s > s0 && !PF)
                load_sub(s, kr, vr);
            if (PF && s + 1 < s1)
                load_sub(s + 1, kn, vn);
            const int key0 = s * kSKeys, nk = min(kSKeys, n - key0);
            const int tn = has_new && s == nsub - 1 ? pos - key0 : -1;
            // scores: four threads per key, a quarter of the dimensions each
            float dot = 0.0f;
            if (kt == tn) {
#pragma unroll
                for (int i = 0; i < KQ; ++i)
                    dot = fmaf(Qs[kq * KQ + i], Kn[kq * KQ + i], dot);
            } else {
#pragma unroll
                for (int i = 0; i < KQ; ++i)
                    dot = fmaf(Qs[kq * KQ + i], s_row_elem<KV, KB>(kr, i), dot);
            }
            dot += __shfl_xor_sync(0xffffffffu, dot, 1);
            if (at && kq == 0)
                Ss[kt] = kt < nk ? dot * a.scale : -INFINITY;
            s_bar();
            if (warp == 0) {
                const float x0 = Ss[lane], x1 = Ss[lane + 32];
                const float mx = warp_max(fmaxf(x0, x1));
                const float mnew = fmaxf(m_run, mx);
                const float p0 = lane < nk ? expf(x0 - mnew) : 0.0f;
                const float p1 = lane + 32 < nk ? expf(x1 - mnew) : 0.0f;
                const float lsub = warp_sum(p0 + p1);
                const float alpha = expf(m_run - mnew);
                l_run = fmaf(l_run, alpha, lsub);
                m_run = mnew;
                Ps[lane] = p0;
                Ps[lane + 32] = p1;
                if (lane == 0)
                    st[0] = alpha;
            }
            s_bar();
            float o0 = 0.0f, o1 = 0.0f;
#pragma unroll
            for (int i = 0; i < VK; ++i) {
                const int t = at ? vg + VG * i : 0;
                const float p = Ps[t];
                float v0, v1;
                if (t == tn) {
                    v0 = Vn[2 * vd];
                    v1 = Vn[2 * vd + 1];
                } else {
                    v0 = s_row_elem<KV, VB>(vr[i], 0);
                    v1 = s_row_elem<KV, VB>(vr[i], 1);
                }
                o0 = fmaf(p, v0, o0);
                o1 = fmaf(p, v1, o1);
            }
            if (at) {
                opart[vg * HD + 2 * vd] = o0;
                opart[vg * HD + 2 * vd + 1] = o1;
            }
            s_bar();
            if (ctid < HD) {
                float t = 0.0f;
#pragma unroll
                for (int w = 0; w < VG; ++w)
                    t += opart[w * HD + ctid];
                o_run = fmaf(o_run, st[0], t);
            }
            if (PF && s + 1 < s1) {
                kr = kn;
#pragma unroll
                for (int i = 0; i < VK; ++i)
                    vr[i] = vn[i];
            }
        }
        u64* pp = part + (size_t)(h * J + j) * (HD + 2);
        if (ctid == 0) {
            ll_putf(pp, m_run, tag);
            ll_putf(pp + 1, l_run, tag);
        }
        if (ctid < HD)
            ll_putf(pp + 2 + ctid, o_run, tag);
        s_bar();  // the scratch is reused by the next item
    }
}

// ---- consumers: GEMV pieces ----------------------------------------------------------------------------

// Sum across the 32 lanes of V values at once (V a power of two <= 32). Each level halves the values a
// lane holds: a lane keeps the half selected by its lane bit and sends the other half to its partner,
// so V values take V - 1 + 5 - log2(V) shuffles instead of 5 V. On return every lane holds the total
// of value j = its lane >> (5 - log2(V)).
template <int V>
__device__ __forceinline__ float s_reduce_lanes(float (&v)[V], int lane)
{
#pragma unroll
    for (int n = V, o = 16; n > 1; n >>= 1, o >>= 1) {
        const bool upper = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < n / 2; ++i) {
            const float send = upper ? v[i] : v[i + n / 2];
            const float keep = upper ? v[i + n / 2] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
    float t = v[0];
#pragma unroll
    for (int o = 32 / V / 2; o >= 1; o >>= 1)
        t += __shfl_xor_sync(0xffffffffu, t, o);
    return t;
}

// out[m][r] = sum over chunks c in [c0, c1) of W_m[row r][8c .. 8c+7] . x[8c .. 8c+7] for R rows of NMAT
// matrices (row r of matrix m at wrow + m * matb + r * rowb in shared memory), every lane getting every
// sum. Lanes take chunks c0 + lane + 32 i, U chunks of every row in flight, one accumulator chain per
// (matrix, row, chunk slot); x (split layout at xs_s) is loaded once per chunk for all rows.
template <int NMAT, int R, int U>
__device__ __forceinline__ void s_dot_rows(unsigned wrow, unsigned rowb, unsigned matb, unsigned xs_s, int K8, int c0,
                                           int c1, int lane, float (&out)[NMAT][R])
{
    constexpr int V = NMAT * R;
    float acc[V][U];
#pragma unroll
    for (int j = 0; j < V; ++j)
#pragma unroll
        for (int u = 0; u < U; ++u)
            acc[j][u] = 0.0f;
    const unsigned xhi = xs_s + 16u * (unsigned)K8;
#pragma unroll 1
    for (int c = c0 + lane; c < c1; c += 32 * U) {
        uint4 w[V][U];
        float4 xa[U], xb[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const unsigned cc = (unsigned)(c + 32 * u);
            if ((int)cc < c1) {
#pragma unroll
                for (int m = 0; m < NMAT; ++m)
#pragma unroll
                    for (int r = 0; r < R; ++r)
                        w[m * R + r][u] = lds_u4(wrow + (unsigned)m * matb + (unsigned)r * rowb + 16u * cc);
                xa[u] = lds_f4(xs_s + 16u * cc);
                xb[u] = lds_f4(xhi + 16u * cc);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (c + 32 * u < c1) {
#pragma unroll
                for (int j = 0; j < V; ++j)
                    acc[j][u] = dot_chunk(w[j][u], xa[u], xb[u], acc[j][u]);
            }
        }
    }
    float v[V];
#pragma unroll
    for (int j = 0; j < V; ++j) {
        float t = acc[j][0];
#pragma unroll
        for (int u = 1; u < U; ++u)
            t += acc[j][u];
        v[j] = t;
    }
    const float mine = s_reduce_lanes<V>(v, lane);
#pragma unroll
    for (int j = 0; j < V; ++j)
        out[j / R][j % R] = __shfl_sync(0xffffffffu, mine, j * (32 / V));
}

// out[m] = sum over chunks c in [c0, c1) of W_m[row][8c .. 8c+7] . x[8c .. 8c+7], the range walked as two
// halves at once (two independent chains per matrix, each with its own x), every lane getting every
// sum. Matrix m's row starts at wrow + m * matb.
template <int NMAT>
__device__ __forceinline__ void s_dot_halves(unsigned wrow, unsigned matb, unsigned xs_s, int K8, int c0, int c1,
                                             int lane, float (&out)[NMAT])
{
    const int h = (c1 - c0 + 1) / 2;  // chunks of the first half
    float acc[NMAT][2];
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
        acc[m][0] = acc[m][1] = 0.0f;
    const unsigned xhi = xs_s + 16u * (unsigned)K8;
#pragma unroll 1
    for (int c = c0 + lane; c < c0 + h; c += 32) {
        const unsigned ca = (unsigned)c, cb = (unsigned)(c + h);
        const bool second = (int)cb < c1;
        uint4 wa[NMAT], wb[NMAT];
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
            wa[m] = lds_u4(wrow + (unsigned)m * matb + 16u * ca);
            if (second)
                wb[m] = lds_u4(wrow + (unsigned)m * matb + 16u * cb);
        }
        const float4 xa0 = lds_f4(xs_s + 16u * ca), xa1 = lds_f4(xhi + 16u * ca);
        float4 xb0 = make_float4(0.f, 0.f, 0.f, 0.f), xb1 = xb0;
        if (second) {
            xb0 = lds_f4(xs_s + 16u * cb);
            xb1 = lds_f4(xhi + 16u * cb);
        }
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
            acc[m][0] = dot_chunk(wa[m], xa0, xa1, acc[m][0]);
            if (second)
                acc[m][1] = dot_chunk(wb[m], xb0, xb1, acc[m][1]);
        }
    }
    float v[NMAT];
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
        v[m] = acc[m][0] + acc[m][1];
    const float mine = s_reduce_lanes<NMAT>(v, lane);
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
        out[m] = __shfl_sync(0xffffffffu, mine, m * (32 / NMAT));
}

struct SBest {
    float v;
    int i;
};

// The pieces of one phase for this CTA, in the producer's order: dot products from the ring, then
// the phase's epilogue for each row:
//   QKV   out = W x + bias           O    out = h (hraw) + W x
//   GU    out = silu(Wg x) * (Wu x)  DOWN out = h1 (h1raw) + W x
//   HEAD  logits[row] = W x, and the thread's best (value, first index)
// Layer phases: a warp per (row, K range), the range walked as two halves at once, a piece of n < 7
// rows split into 7 / n K ranges whose partial sums are added in a fixed order; the LM head: two rows
// per warp (w and w + 7 of a piece).
template <int PH>
__device__ __forceinline__ void s_consume(const SArgs& a, SRing& pos, u64& idx, int l, u64* out, unsigned tag, int ctid,
                                       SBest& best)
{
    extern __shared__ __align__(128) char smem[];
    const SSmem S = s_smem(a, smem, a.heads);
    constexpr int NMAT = PH == SP_GU ? 2 : 1;
    const SGeom g = s_geom(a, l, PH);
    const unsigned R = (unsigned)a.ring_bytes;
    const int K8 = g.K / 8;
    const unsigned ring_s = smem_u32(S.ring), xs_s = smem_u32(S.xs);
    const int warp = ctid >> 5, lane = ctid & 31;
    // Fields of the kernel argument used per row, read once (the stores below could alias them).
    const float* bias = nullptr;
    if constexpr (PH == SP_QKV)
        bias = a.layers[l].bqkv;
    float* const logits = a.logits;
    const float* const hraw = S.hraw;
    const float* const h1raw = S.h1raw;
    uint64_t* const full = S.full;
    uint64_t* const empty = S.empty;
    auto epilogue = [&](int row, float v0, float v1) {
        if (PH == SP_QKV)
            ll_putf(out + row, v0 + __ldg(bias + row), tag);
        else if (PH == SP_O)
            ll_putf(out + row, hraw[row] + v0, tag);
        else if (PH == SP_GU)
            ll_putf(out + row, silu_mul(v0, v1), tag);
        else if (PH == SP_DOWN)
            ll_putf(out + row, h1raw[row] + v0, tag);
        else {
            logits[row] = v0;
            if (pair_better(v0, row, best.v, best.i))
                best.v = v0, best.i = row;
        }
    };
    int pc = 0;
#pragma unroll 1
    for (int r0 = g.rb; r0 < g.re; r0 += g.rpp, ++pc) {
        const int n = min(g.rpp, g.re - r0);
        const unsigned part = (unsigned)n * (unsigned)g.K * 2u;
        unsigned phys;
        s_place(pos, s_round128(part * NMAT), R, phys);
        const u64 t = idx++;
        const bool have = s_wait(a, &full[t % kSBars], (unsigned)((t / kSBars) & 1));
        const unsigned base = ring_s + phys, rowb = (unsigned)g.K * 2u;
        if constexpr (PH == SP_HEAD) {
#pragma unroll 1
            for (int r = warp; r < n; r += 2 * kSWarps) {
                const int r1 = r + kSWarps < n ? r + kSWarps : r;  // a missing second row repeats the first
                float acc[1][2] = {{0.0f, 0.0f}};
                if (have)
                    s_dot_rows<1, 2, 2>(base + (unsigned)r * rowb, (unsigned)(r1 - r) * rowb, 0u, xs_s, K8, 0, K8,
                                        lane, acc);
                if (lane == 0) {
                    epilogue(r0 + r, acc[0][0], 0.0f);
                    if (r1 != r)
                        epilogue(r0 + r1, acc[0][1], 0.0f);
                }
            }
            __syncwarp();
            if (have && lane == 0)
                mbar_arrive(&empty[t % kSBars]);
            continue;
        }
        const int KS = n < kSWarps ? kSWarps / n : 1;
        float* psum = S.psum + (pc & 1) * 128;  // [m][64]
#pragma unroll 1
        for (int u = warp; u < n * KS; u += kSWarps) {
            const int r = u / KS, sg = u % KS;
            float acc[NMAT];
#pragma unroll
            for (int m = 0; m < NMAT; ++m)
                acc[m] = 0.0f;
            if (have)
                s_dot_halves<NMAT>(base + (unsigned)r * rowb, part, xs_s, K8, K8 * sg / KS, K8 * (sg + 1) / KS, lane,
                                   acc);
            if (KS == 1) {
                if (lane == 0)
                    epilogue(r0 + r, acc[0], acc[NMAT - 1]);
            } else if (lane == 0) {
#pragma unroll
                for (int m = 0; m < NMAT; ++m)
                    psum[m * 64 + u] = acc[m];
            }
        }
        __syncwarp();
        if (have && lane == 0)
            mbar_arrive(&empty[t % kSBars]);
        if (KS > 1) {
            s_bar();
            for (int r = ctid; r < n; r += kSCThreads) {
                float v[NMAT];
#pragma unroll
                for (int m = 0; m < NMAT; ++m) {
                    float x = 0.0f;
                    for (int q = 0; q < KS; ++q)
                        x += psum[m * 64 + r * KS + q];
                    v[m] = x;
                }
                epilogue(r0 + r, v[0], v[NMAT - 1]);
            }
        }
    }
}

// ---- the kernel ----------------------------------------------------------------------------------------

template <typename KV, int HD>
__global__ void __launch_bounds__(kSThreads, 1) k_decode_stream(const __grid_constant__ SArgs a)
{
    extern __shared__ __align__(128) char smem[];
    const SSmem S = s_smem(a, smem, a.heads);
    if (threadIdx.x == 0) {
        for (int s = 0; s < kSBars; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], kSWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x >= kSCThreads) {
        if (threadIdx.x == kSCThreads)
            s_producer(a);
        return;
    }

    const int ctid = threadIdx.x, warp = ctid >> 5, lane = ctid & 31;
    const int H = a.H, G = gridDim.x;
    SRing rpos{0, 0};
    u64 idx = 0;
    int next_tok = 0;
    for (int k = 0; k < a.n_steps; ++k) {
        const unsigned tag = a.tag0 + (unsigned)k;
        const int pos = min(a.pos0 + k, a.max_seq - 1);
        int token = a.pos0 + k < a.prompt_end ? __ldcg(a.tokens + pos) : next_tok;
        if (token < 0 || token >= a.V)
            token = 0;
        const int nsub = (pos + kSKeys) / kSKeys, J = min(nsub, kSJmax);
        SBest best{-INFINITY, INT_MAX};
        for (int l = 0; l < a.L; ++l) {
            const SLayer& Ly = a.layers[l];
            u64* blk = a.ll + (size_t)l * a.ll_layer;
            // QKV: the layer input (layer 0: the embedding row of the token) into hraw, rms_norm -> xs
            if (l == 0) {
                const __half2* e = reinterpret_cast<const __half2*>(a.embd + (size_t)token * H);
                for (int q = ctid; q < H / 2; q += kSCThreads)
                    reinterpret_cast<float2*>(S.hraw)[q] = __half22float2(__ldg(e + q));
            } else {
                const u64* src = a.ll + (size_t)(l - 1) * a.ll_layer + a.o_hout;
                s_poll(a, src, H, tag, ctid,
                       [&](int q, float v0, float v1) { reinterpret_cast<float2*>(S.hraw)[q] = make_float2(v0, v1); });
            }
            s_norm(S.hraw, Ly.attn_norm, a.eps, H, S.xs, S.red, ctid);
            s_consume<SP_QKV>(a, rpos, idx, l, blk + a.o_qkv, tag, ctid, best);
            // attention items of this CTA, then the O projection's input: the merged partials
            s_attention<KV, HD>(a, l, pos, J, tag, ctid);
            s_merge<HD>(a, blk + a.o_part, J, tag, ctid);
            s_consume<SP_O>(a, rpos, idx, l, blk + a.o_h1, tag, ctid, best);
            // gate/up: h1 into h1raw, rms_norm -> xs
            s_poll(a, blk + a.o_h1, H, tag, ctid,
                   [&](int q, float v0, float v1) { reinterpret_cast<float2*>(S.h1raw)[q] = make_float2(v0, v1); });
            s_norm(S.h1raw, Ly.ffn_norm, a.eps, H, S.xs, S.red, ctid);
            s_consume<SP_GU>(a, rpos, idx, l, blk + a.o_act, tag, ctid, best);
            // down: the SwiGLU output straight into xs (after every warp is done with the gate/up input)
            s_bar();
            {
                const int K8 = a.F / 8;
                s_poll(a, blk + a.o_act, a.F, tag, ctid, [&](int q, float v0, float v1) {
                    *reinterpret_cast<float2*>(S.xs + xs_index(2 * q, K8)) = make_float2(v0, v1);
                });
            }
            s_bar();
            s_consume<SP_DOWN>(a, rpos, idx, l, blk + a.o_hout, tag, ctid, best);
        }
        // LM head: final rms_norm -> logits, this CTA's best
        s_poll(a, a.ll + (size_t)(a.L - 1) * a.ll_layer + a.o_hout, H, tag, ctid,
               [&](int q, float v0, float v1) { reinterpret_cast<float2*>(S.hraw)[q] = make_float2(v0, v1); });
        s_norm(S.hraw, a.final_norm, a.eps, H, S.xs, S.red, ctid);
        s_consume<SP_HEAD>(a, rpos, idx, a.L, nullptr, tag, ctid, best);
        // Greedy pick (src/Sampler.cpp:32-43, the first index of the maximum) over every CTA's best.
        warp_argmax(best.v, best.i);
        if (lane == 0) {
            S.bestv[warp] = best.v;
            S.besti[warp] = best.i;
        }
        s_bar();
        u64* bw = a.ll_best + (size_t)(k & 1) * 2 * G;
        if (warp == 0) {
            float v = lane < kSWarps ? S.bestv[lane] : -INFINITY;
            int i = lane < kSWarps ? S.besti[lane] : INT_MAX;
            warp_argmax(v, i);
            if (lane == 0) {
                __threadfence();  // this CTA's cache rows (fenced by their writers) before its pair
                ll_putf(bw + 2 * blockIdx.x, v, tag);
                ll_put(bw + 2 * blockIdx.x + 1, (unsigned)i, tag);
            }
        }
        {
            float v = -INFINITY;
            int i = INT_MAX;
            for (int q = ctid; q < G; q += kSCThreads) {
                u64 w0 = 0, w1 = 0;
                unsigned long long t0 = 0;
                for (int it = 1;; ++it) {
                    ll_get2(bw + 2 * q, w0, w1);
                    if (ll_tag(w0) == tag && ll_tag(w1) == tag)
                        break;
                    if ((it & 7) == 0) {
                        if (s_aborted(a))
                            break;
                        if (t0 == 0)
                            t0 = now_ns();
                        else if (now_ns() - t0 > kWaitLimitNs) {
                            s_fail(a);
                            break;
                        }
                    }
                }
                const float qv = ll_val(w0);
                const int qi = (int)(unsigned)w1;
                if (pair_better(qv, qi, v, i))
                    v = qv, i = qi;
            }
            __threadfence();  // acquire side: the other CTAs' cache rows before the next step reads them
            warp_argmax(v, i);
            s_bar();
            if (lane == 0) {
                S.bestv[warp] = v;
                S.besti[warp] = i;
            }
            s_bar();
            if (warp == 0) {
                float vv = lane < kSWarps ? S.bestv[lane] : -INFINITY;
                int ii = lane < kSWarps ? S.besti[lane] : INT_MAX;
                warp_argmax(vv, ii);
                if (lane == 0)
                    S.greedy[0] = ii == INT_MAX ? 0 : ii;
            }
            s_bar();
        }
        const int greedy = S.greedy[0];
        const int p1 = a.pos0 + k + 1;
        next_tok = p1 < a.prompt_end && p1 < a.max_seq ? __ldcg(a.tokens + p1) : greedy;
        if (blockIdx.x == 0 && ctid == 0) {
            if (p1 >= a.prompt_end && p1 < a.total && p1 < a.max_seq)
                a.tokens[p1] = greedy;
            a.ctrl->greedy = greedy;
            a.ctrl->step = p1;
        }
    }
}

}  // namespace muyo
