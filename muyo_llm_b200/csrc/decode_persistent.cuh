// The persistent decode kernel: every decode step of a generate call in ONE cooperative launch,
// one CTA per SM.
//
// Why: at batch 1 a Qwen2.5-0.5B step is ~120 dependent GEMV/attention phases of 0.3-3 us of HBM time
// each; as separate kernels each phase pays a launch and a chain of dependent global round trips
// (stage x -> norm -> weight fetch -> reduce), which measured 4-10x its HBM time. Here the weights,
// which do not depend on the activations, are streamed ahead of the activation dependencies:
//
//   warp 0 (producer)  walks the static schedule of every weight tile this SM consumes in the whole
//                      generate call (layer by layer, phase by phase, then the LM head, step after
//                      step) and copies each tile global -> shared memory with cp.async.bulk into a
//                      ring of slots, each slot guarded by a full/empty mbarrier pair. It runs ahead
//                      across phase boundaries and grid barriers, bounded only by the ring.
//   warps 1..11        run the phases; between phases they meet at a grid barrier (one global
//   (consumers)        arrival counter, acquire spin). Per layer:
//                        QKV    x = rms_norm(h) (layer 0: the embedding row of the fed token) -> W_qkv x + b
//                        ATTN   RoPE + KV append + split-K GQA attention partials (attention_item)
//                        O      merge the partials -> h1 = h + W_o attn
//                        GATEUP x = rms_norm(h1) -> act = silu(W_gate x) * (W_up x)
//                        DOWN   h = h1 + W_down act
//                      then HEAD: logits = W_out rms_norm(h), the greedy pick, and the next token.
//
// Rows of every matrix are split into one contiguous range per CTA; a warp takes two rows of a tile
// at a time, its lanes the 16-byte chunks of those rows in shared memory, x in shared memory in the
// split layout of gemv.cuh. Activations written within the launch are read with ld.global.cg (L2),
// never through L1. Every wait (mbarrier or grid barrier) is bounded by the global timer: on expiry
// the CTA records MUYO_ETIMEOUT in the error word, stops, drains its own copies and returns.
#pragma once

#include "attention.cuh"
#include "common.cuh"
#include "gemv.cuh"

namespace muyo {

constexpr int kPWarps = 8;
constexpr int kPThreads = kPWarps * 32;
constexpr int kCWarps = kPWarps - 1;
constexpr int kCThreads = kCWarps * 32;
constexpr int kMaxSlots = 8;
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s per wait

struct PLayer {
    const __half* wqkv;
    const float* bqkv;
    const float* attn_norm;
    const __half* wo;
    const float* ffn_norm;
    const __half* wgate;
    const __half* wup;
    const __half* wdown;
};

struct PArgs {
    const PLayer* layers;
    int L;
    const __half* embd;
    const __half* lm;
    const float* final_norm;
    int H, F, V, QKV, QD, KVD, heads, kv_heads, gqa, hd, max_seq;
    float eps;
    AttnDev attn;
    void* kc;
    void* vc;
    long long kv_layer_elems;
    float* h;
    float* h1;
    float* qkv;
    float* act;
    float* logits;
    float* attn_part;
    Pair* lm_part;
    Control* ctrl;
    int32_t* tokens;
    unsigned* bar;
    int* err;
    int n_steps;
    int slots, slot_bytes, region_b_bytes;
};

enum PPhase { PH_QKV = 0, PH_O = 1, PH_GATEUP = 2, PH_DOWN = 3, PH_HEAD = 4 };

struct TileGeom {
    const __half* w0;
    const __half* w1;
    int rows, K, nmat;
};

__device__ __forceinline__ TileGeom phase_geom(const PArgs& a, int layer, int ph)
{
    if (ph == PH_HEAD)
        return TileGeom{a.lm, nullptr, a.V, a.H, 1};
    const PLayer& L = a.layers[layer];
    switch (ph) {
        case PH_QKV: return TileGeom{L.wqkv, nullptr, a.QKV, a.H, 1};
        case PH_O: return TileGeom{L.wo, nullptr, a.H, a.QD, 1};
        case PH_GATEUP: return TileGeom{L.wgate, L.wup, a.F, a.H, 2};
        default: return TileGeom{L.wdown, nullptr, a.H, a.F, 1};
    }
}

__device__ __forceinline__ unsigned smem_u32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }

__device__ __forceinline__ unsigned long long now_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* b, unsigned count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, unsigned bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* b)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, unsigned parity)
{
    unsigned ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase of `b` with the given parity; false (and the abort flag set) on expiry
// or when another warp of the CTA aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, unsigned parity, volatile int* abort_sm)
{
    if (mbar_try_wait(b, parity))
        return true;
    const unsigned long long t0 = now_ns();
    while (true) {
        if (mbar_try_wait(b, parity))
            return true;
        if (*abort_sm)
            return false;
        if (now_ns() - t0 > kWaitLimitNs) {
            *abort_sm = 1;
            return false;
        }
    }
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"r"(kCThreads) : "memory"); }

struct ConsumerSync {
    __device__ __forceinline__ void operator()() const { consumer_sync(); }
};

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p)
{
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid barrier among the consumer warps of all CTAs (the producer never joins). `k` counts the
// barriers of this launch; the counter was zeroed before the launch. The named barrier orders the
// CTA's writes before thread 0's acq_rel fence and relaxed arrival (the release pattern of a GPU-scope
// barrier); the acquire poll orders the reads that follow.
__device__ __forceinline__ bool grid_sync(const PArgs& a, unsigned& k, int ctid, volatile int* abort_sm)
{
    ++k;
    consumer_sync();
    if (ctid == 0 && !*abort_sm) {
        const unsigned target = k * gridDim.x;
        asm volatile("fence.acq_rel.gpu;\n\tred.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(a.bar) : "memory");
        if (ld_acquire_u32(a.bar) < target) {
            const unsigned long long t0 = now_ns();
            while (ld_acquire_u32(a.bar) < target) {
                if (now_ns() - t0 > kWaitLimitNs) {
                    *abort_sm = 1;
                    break;
                }
            }
        }
    }
    consumer_sync();
    return !*abort_sm;
}

// Rows [rb, re) of an M-row matrix owned by this CTA, and the rows per tile for this geometry.
__device__ __forceinline__ void cta_rows(int M, int& rb, int& re)
{
    rb = (int)((long long)M * blockIdx.x / gridDim.x);
    re = (int)((long long)M * (blockIdx.x + 1) / gridDim.x);
}

__device__ __forceinline__ int tile_rows(const PArgs& a, const TileGeom& g)
{
    return a.slot_bytes / (g.K * 2 * g.nmat);
}

// Tiles of one phase for this CTA: its rows [rb, re) split evenly into ceil(rows / R) tiles
// (R rows fit a slot), so no tile is a small remainder.
__device__ __forceinline__ void tile_span(int rb, int re, int R, int t, int& r0, int& n, int& ntiles)
{
    const int rows = re - rb;
    ntiles = rows > 0 ? (rows + R - 1) / R : 0;
    if (ntiles == 0) {
        r0 = rb;
        n = 0;
        return;
    }
    const int a = rows * t / ntiles, b = rows * (t + 1) / ntiles;  // rows per CTA stay far below 2^31 / ntiles
    r0 = rb + a;
    n = b - a;
}

// ---- producer ---------------------------------------------------------------------------------------

__device__ void producer_loop(const PArgs& a, char* ring, uint64_t* full, uint64_t* empty, volatile int* abort_sm)
{
    unsigned long long i = 0;
    for (int step = 0; step < a.n_steps && !*abort_sm; ++step) {
        for (int l = 0; l <= a.L && !*abort_sm; ++l) {
            const int nph = l < a.L ? 4 : 1;
            for (int q = 0; q < nph && !*abort_sm; ++q) {
                const int ph = l < a.L ? q : PH_HEAD;
                const TileGeom g = phase_geom(a, l, ph);
                int rb, re;
                cta_rows(g.rows, rb, re);
                const int R = tile_rows(a, g);
                int ntiles = 1;
                for (int t = 0; t < ntiles; ++t, ++i) {
                    int r0, n;
                    tile_span(rb, re, R, t, r0, n, ntiles);
                    if (ntiles == 0)
                        break;
                    const int s = (int)(i % a.slots);
                    if (i >= (unsigned long long)a.slots &&
                        !mbar_wait(&empty[s], (unsigned)(((i / a.slots) - 1) & 1), abort_sm))
                        break;
                    const unsigned part = (unsigned)n * g.K * 2;
                    char* dst = ring + (size_t)s * a.slot_bytes;
                    mbar_expect_tx(&full[s], part * g.nmat);
                    bulk_g2s(dst, g.w0 + (size_t)r0 * g.K, part, &full[s]);
                    if (g.nmat == 2)
                        bulk_g2s(dst + part, g.w1 + (size_t)r0 * g.K, part, &full[s]);
                }
            }
        }
    }
    // Drain: every copy issued into a slot must land before the CTA may exit. The last use of each
    // slot is the most recent phase of its full barrier.
    const unsigned long long issued = i;
    for (unsigned long long k = issued > (unsigned long long)a.slots ? issued - a.slots : 0; k < issued; ++k) {
        const int s = (int)(k % a.slots);
        const unsigned long long t0 = now_ns();
        while (!mbar_try_wait(&full[s], (unsigned)((k / a.slots) & 1)) && now_ns() - t0 < kWaitLimitNs) {
        }
    }
}

// ---- consumers -----------------------------------------------------------------------------------------

// Stage a K-vector into xs (split layout of gemv.cuh). NORM applies x / sqrt(mean(x^2) + eps) * w
// (tools/reference_qwen2.py:81-82). EMBED reads row `token` of the F16 table, and CTA 0 also stores
// it to `copy` (the residual stream). All loads (x and w) are issued before any is used: one L2 round
// trip per phase. K must be a multiple of 8.
template <bool NORM, bool EMBED>
__device__ __noinline__ void stage_x(const float* src, const __half* erow, const float* w, float eps, int K,
                                        float* xs, float* red, float* copy, int ctid)
{
    constexpr int NB = 2;  // 8-element chunks per thread per pass
    const int K8 = K / 8;
    float ss = 0.0f;
    for (int base = 0; base < K8; base += NB * kCThreads) {
        float4 lo[NB], hi[NB], wl[NB], wh[NB];
#pragma unroll
        for (int u = 0; u < NB; ++u) {
            const int c = base + u * kCThreads + ctid;
            if (c < K8) {
                if (EMBED) {
                    const uint4 hv = __ldg(reinterpret_cast<const uint4*>(erow) + c);
                    const float2 a0 = h2_to_f2(hv.x), a1 = h2_to_f2(hv.y), a2 = h2_to_f2(hv.z), a3 = h2_to_f2(hv.w);
                    lo[u] = make_float4(a0.x, a0.y, a1.x, a1.y);
                    hi[u] = make_float4(a2.x, a2.y, a3.x, a3.y);
                } else {
                    lo[u] = __ldcg(reinterpret_cast<const float4*>(src) + 2 * c);
                    hi[u] = __ldcg(reinterpret_cast<const float4*>(src) + 2 * c + 1);
                }
                if (NORM) {
                    wl[u] = __ldg(reinterpret_cast<const float4*>(w) + 2 * c);
                    wh[u] = __ldg(reinterpret_cast<const float4*>(w) + 2 * c + 1);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < NB; ++u) {
            const int c = base + u * kCThreads + ctid;
            if (c < K8) {
                if (NORM) {
                    ss = fmaf(lo[u].x, lo[u].x, ss); ss = fmaf(lo[u].y, lo[u].y, ss);
                    ss = fmaf(lo[u].z, lo[u].z, ss); ss = fmaf(lo[u].w, lo[u].w, ss);
                    ss = fmaf(hi[u].x, hi[u].x, ss); ss = fmaf(hi[u].y, hi[u].y, ss);
                    ss = fmaf(hi[u].z, hi[u].z, ss); ss = fmaf(hi[u].w, hi[u].w, ss);
                    // keep raw x and w side by side until the scale is known
                    reinterpret_cast<float4*>(xs)[c] = lo[u];
                    reinterpret_cast<float4*>(xs + 4 * K8)[c] = hi[u];
                    reinterpret_cast<float4*>(xs + 8 * K8)[c] = wl[u];
                    reinterpret_cast<float4*>(xs + 12 * K8)[c] = wh[u];
                } else {
                    reinterpret_cast<float4*>(xs)[c] = lo[u];
                    reinterpret_cast<float4*>(xs + 4 * K8)[c] = hi[u];
                }
                if (EMBED && blockIdx.x == 0) {
                    reinterpret_cast<float4*>(copy)[2 * c] = lo[u];
                    reinterpret_cast<float4*>(copy)[2 * c + 1] = hi[u];
                }
            }
        }
    }
    if (!NORM) {
        consumer_sync();
        return;
    }
    ss = warp_sum(ss);
    const int lane = ctid & 31, warp = ctid >> 5;
    if (lane == 0)
        red[warp] = ss;
    consumer_sync();
    float t = lane < kCWarps ? red[lane] : 0.0f;
    t = warp_sum(t);
    const float s = __fsqrt_rn(__fdiv_rn(t, (float)K) + eps);
#pragma unroll 1
    for (int i = ctid; i < 8 * K8; i += kCThreads)
        xs[i] = __fdiv_rn(xs[i], s) * xs[8 * K8 + i];
    consumer_sync();
}

struct HeadBest {
    float v;
    int i;
};

__device__ __forceinline__ uint4 lds_u4(unsigned addr)
{
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}

__device__ __forceinline__ float4 lds_f4(unsigned addr)
{
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}

// Dot products of NR rows (of NMAT matrices; NR * NMAT = 2 dot products) of a tile with x, for one
// lane: the lane takes the 16-byte chunks c = lane + 32 j; four chunks are loaded before any is used
// and accumulate into four independent chains per dot product (instruction-level parallelism over
// the shared-memory latency). All operands are read with ld.shared from 32-bit shared addresses
// (the tile at `base`, the split-layout x at `xs`), which stays explicit across the out-of-line
// phase functions.
template <int NMAT, int NR>
__device__ __forceinline__ void dot_rows(unsigned base, unsigned rowb, unsigned matb, int ra, int rb_, int K8,
                                         unsigned xs, int lane, float (&out)[NMAT][2])
{
    static_assert(NMAT * NR == 2, "two dot products per pass");
    float acc[NMAT][NR][4];
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int j = 0; j < NR; ++j)
#pragma unroll
            for (int q = 0; q < 4; ++q)
                acc[m][j][q] = 0.0f;
    unsigned w[NMAT][NR];
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
        w[m][0] = base + m * matb + ra * rowb;
        if (NR > 1)
            w[m][NR - 1] = base + m * matb + rb_ * rowb;
    }
    const unsigned xhi = xs + 16u * K8;
    for (int c0 = lane; c0 < K8; c0 += 128) {
        uint4 wv[NMAT][NR][4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int c = c0 + 32 * q;
            if (c < K8) {
#pragma unroll
                for (int m = 0; m < NMAT; ++m)
#pragma unroll
                    for (int j = 0; j < NR; ++j)
                        wv[m][j][q] = lds_u4(w[m][j] + 16u * c);
            }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int c = c0 + 32 * q;
            if (c < K8) {
                const float4 xa = lds_f4(xs + 16u * c), xb = lds_f4(xhi + 16u * c);
#pragma unroll
                for (int m = 0; m < NMAT; ++m)
#pragma unroll
                    for (int j = 0; j < NR; ++j) {
                        const uint4 v = wv[m][j][q];
                        float s = acc[m][j][q];
                        float2 f = h2_to_f2(v.x);
                        s = fmaf(f.x, xa.x, s);
                        s = fmaf(f.y, xa.y, s);
                        f = h2_to_f2(v.y);
                        s = fmaf(f.x, xa.z, s);
                        s = fmaf(f.y, xa.w, s);
                        f = h2_to_f2(v.z);
                        s = fmaf(f.x, xb.x, s);
                        s = fmaf(f.y, xb.y, s);
                        f = h2_to_f2(v.w);
                        s = fmaf(f.x, xb.z, s);
                        s = fmaf(f.y, xb.w, s);
                        acc[m][j][q] = s;
                    }
            }
        }
    }
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int j = 0; j < 2; ++j)
            out[m][j] = j < NR ? warp_sum((acc[m][j < NR ? j : 0][0] + acc[m][j < NR ? j : 0][1]) +
                                          (acc[m][j < NR ? j : 0][2] + acc[m][j < NR ? j : 0][3]))
                               : 0.0f;
}

// Consume this CTA's tiles of one phase: two rows per warp pass, lanes over 16-byte chunks.
template <int EPI>
__device__ __noinline__ void consume_phase(const PArgs& a, const TileGeom& g, const float* xs, char* ring,
                                              uint64_t* full, uint64_t* empty, unsigned long long& ti, int layer,
                                              int cwarp, int lane, volatile int* abort_sm, HeadBest& best)
{
    constexpr int NMAT = EPI == PH_GATEUP ? 2 : 1;
    int rb, re;
    cta_rows(g.rows, rb, re);
    const int R = tile_rows(a, g);
    const int K8 = g.K / 8;
    const unsigned xs_s = smem_u32(xs), ring_s = smem_u32(ring);
    const PLayer* L = layer < a.L ? &a.layers[layer] : nullptr;
    int ntiles = 1;
    for (int t = 0; t < ntiles; ++t, ++ti) {
        int r0, n;
        tile_span(rb, re, R, t, r0, n, ntiles);
        if (ntiles == 0)
            break;
        const int s = (int)(ti % a.slots);
        if (!mbar_wait(&full[s], (unsigned)((ti / a.slots) & 1), abort_sm))
            continue;  // aborted: skip this warp's work (no barrier is skipped)
        const unsigned base = ring_s + (unsigned)s * a.slot_bytes;
        const unsigned rowb = (unsigned)g.K * 2, matb = (unsigned)n * rowb;
        constexpr int NR = 2 / NMAT;  // rows per warp pass
        for (int r = NR * cwarp; r < n; r += NR * kCWarps) {
            const bool two = NR == 2 && r + 1 < n;
            // epilogue operands, loaded before the dot products so their latency overlaps them
            float pre[2] = {0.f, 0.f};
            if (lane == 0) {
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int row = r0 + (j == 1 && two ? r + 1 : r);
                    if (EPI == PH_QKV)
                        pre[j] = __ldg(L->bqkv + row);
                    else if (EPI == PH_O)
                        pre[j] = __ldcg(a.h + row);
                    else if (EPI == PH_DOWN)
                        pre[j] = __ldcg(a.h1 + row);
                }
            }
            float acc[NMAT][2];
            dot_rows<NMAT, NR>(base, rowb, matb, r, two ? r + 1 : r, K8, xs_s, lane, acc);
            if (lane == 0) {
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    if (j == 1 && !two)
                        break;
                    const int row = r0 + r + j;
                    const float v = acc[0][j];
                    if (EPI == PH_QKV) {
                        a.qkv[row] = v + pre[j];
                    } else if (EPI == PH_O) {
                        a.h1[row] = pre[j] + v;
                    } else if (EPI == PH_GATEUP) {
                        a.act[row] = silu_mul(v, acc[NMAT - 1][0]);
                    } else if (EPI == PH_DOWN) {
                        a.h[row] = pre[j] + v;
                    } else {
                        a.logits[row] = v;
                        if (pair_better(v, row, best.v, best.i))
                            best.v = v, best.i = row;
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0)
            mbar_arrive(&empty[s]);
    }
}

// The attention work items of this CTA at `pos` (one layer), then the O-phase input: the merged
// attention output staged into xs. The phases are out of line so that each gets its own register
// allocation (the whole step inlined into one loop body exceeds 255 registers).
template <typename KV, int HD>
__device__ __noinline__ void attention_phase(const PArgs& a, int l, int pos, int nchunks, float* region_b, double* cs,
                                             int ctid)
{
    KV* kcl = static_cast<KV*>(a.kc) + (size_t)a.kv_layer_elems * l;
    KV* vcl = static_cast<KV*>(a.vc) + (size_t)a.kv_layer_elems * l;
    for (int it = blockIdx.x; it < a.kv_heads * nchunks; it += gridDim.x) {
        attention_item<KV, HD, true>(a.attn, a.qkv, kcl, vcl, pos, it % a.kv_heads, it / a.kv_heads, nullptr,
                                     a.attn_part, region_b, cs, ctid, kCThreads, ConsumerSync{});
        consumer_sync();
    }
}

template <int HD>
__device__ __noinline__ void merge_phase(const PArgs& a, int nchunks, float* region_b, int ctid)
{
    const int K8 = a.QD / 8;
    float* xs = region_b;
    attn_merge_all<HD>(a.attn, a.attn_part, nchunks, region_b + a.QD, ctid, kCThreads, ConsumerSync{},
                       [&](int e, float v) { xs[xs_index(e, K8)] = v; });
    consumer_sync();
}

template <typename KV, int HD>
__global__ void __launch_bounds__(kPThreads, 1) k_decode_persistent(PArgs a)
{
    extern __shared__ __align__(128) char smem[];
    char* ring = smem;
    float* region_b = reinterpret_cast<float*>(smem + (size_t)a.slots * a.slot_bytes);
    double* cs = reinterpret_cast<double*>(reinterpret_cast<char*>(region_b) + a.region_b_bytes);
    float* red = reinterpret_cast<float*>(cs + HD);
    Pair* bests = reinterpret_cast<Pair*>(red + 32);
    uint64_t* full = reinterpret_cast<uint64_t*>(bests + 32);
    uint64_t* empty = full + kMaxSlots;
    __shared__ int abort_flag;
    volatile int* abort_sm = &abort_flag;

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < a.slots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kCWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (threadIdx.x < 32) {
        if (threadIdx.x == 0)
            producer_loop(a, ring, full, empty, abort_sm);
        if (threadIdx.x == 0 && *abort_sm)
            atomicMax(a.err, -MUYO_ETIMEOUT);
        return;
    }

    // Consumers. Every consumer warp executes the same sequence of named barriers whatever happens:
    // a timed-out wait only skips work local to a warp (and the grid-level spin), never a barrier, so
    // an aborted launch still ends in bounded time.
    const int ctid = threadIdx.x - 32, cwarp = ctid >> 5, lane = ctid & 31;
    unsigned k = 0;
    unsigned long long ti = 0;
    for (int step = 0; step < a.n_steps; ++step) {
        int pos = __ldcg(&a.ctrl->step);
        if (pos < 0 || pos >= a.max_seq) {
            *abort_sm = 1;
            pos = 0;
        }
        int token = __ldcg(a.tokens + pos);
        if (token < 0 || token >= a.V)
            token = 0;
        const int nchunks = (pos + 1 + kAttnKeys - 1) / kAttnKeys;
        HeadBest unused{-INFINITY, INT_MAX};
        for (int l = 0; l < a.L; ++l) {
            const PLayer& Ly = a.layers[l];
            // QKV
            if (l == 0)
                stage_x<true, true>(nullptr, a.embd + (size_t)token * a.H, Ly.attn_norm, a.eps, a.H, region_b, red,
                                    a.h, ctid);
            else
                stage_x<true, false>(a.h, nullptr, Ly.attn_norm, a.eps, a.H, region_b, red, nullptr, ctid);
            consume_phase<PH_QKV>(a, phase_geom(a, l, PH_QKV), region_b, ring, full, empty, ti, l, cwarp, lane,
                                  abort_sm, unused);
            grid_sync(a, k, ctid, abort_sm);
            // ATTN: work items (kv head, chunk) spread over the CTAs
            attention_phase<KV, HD>(a, l, pos, nchunks, region_b, cs, ctid);
            grid_sync(a, k, ctid, abort_sm);
            // O: merge the attention partials straight into the staged x
            merge_phase<HD>(a, nchunks, region_b, ctid);
            consume_phase<PH_O>(a, phase_geom(a, l, PH_O), region_b, ring, full, empty, ti, l, cwarp, lane, abort_sm,
                                unused);
            grid_sync(a, k, ctid, abort_sm);
            // GATE / UP
            stage_x<true, false>(a.h1, nullptr, Ly.ffn_norm, a.eps, a.H, region_b, red, nullptr, ctid);
            consume_phase<PH_GATEUP>(a, phase_geom(a, l, PH_GATEUP), region_b, ring, full, empty, ti, l, cwarp, lane,
                                     abort_sm, unused);
            grid_sync(a, k, ctid, abort_sm);
            // DOWN
            stage_x<false, false>(a.act, nullptr, nullptr, 0.0f, a.F, region_b, red, nullptr, ctid);
            consume_phase<PH_DOWN>(a, phase_geom(a, l, PH_DOWN), region_b, ring, full, empty, ti, l, cwarp, lane,
                                   abort_sm, unused);
            grid_sync(a, k, ctid, abort_sm);
        }
        // HEAD: logits, the CTA's best (value, index), then CTA 0 picks the next token
        stage_x<true, false>(a.h, nullptr, a.final_norm, a.eps, a.H, region_b, red, nullptr, ctid);
        HeadBest best{-INFINITY, INT_MAX};
        consume_phase<PH_HEAD>(a, phase_geom(a, a.L, PH_HEAD), region_b, ring, full, empty, ti, a.L, cwarp, lane,
                               abort_sm, best);
        if (lane == 0)
            bests[cwarp] = Pair{best.v, best.i};
        consumer_sync();
        if (cwarp == 0) {
            Pair p = lane < kCWarps ? bests[lane] : Pair{-INFINITY, INT_MAX};
            warp_argmax(p.v, p.i);
            if (lane == 0)
                a.lm_part[blockIdx.x] = p;
        }
        grid_sync(a, k, ctid, abort_sm);
        if (blockIdx.x == 0 && cwarp == 0) {
            float v = -INFINITY;
            int i = INT_MAX;
            for (int q = lane; q < (int)gridDim.x; q += 32) {
                const float qv = __ldcg(&a.lm_part[q].v);
                const int qi = __ldcg(&a.lm_part[q].i);
                if (pair_better(qv, qi, v, i))
                    v = qv, i = qi;
            }
            warp_argmax(v, i);
            if (lane == 0) {
                const int greedy = i == INT_MAX ? 0 : i;
                Control* c = a.ctrl;
                const int s = __ldcg(&c->step);
                if (s + 1 < __ldcg(&c->total) && s + 1 < a.max_seq) {
                    const int next = s + 1 < __ldcg(&c->prompt_end) ? __ldcg(a.tokens + s + 1) : greedy;
                    a.tokens[s + 1] = next;
                }
                c->greedy = greedy;
                c->step = s + 1;
            }
        }
        grid_sync(a, k, ctid, abort_sm);
    }
    if (ctid == 0 && *abort_sm)
        atomicMax(a.err, -MUYO_ETIMEOUT);
}

}  // namespace muyo
