// The fused decode step: the reference's 18-node Qwen2 layer (src/FullModel.cpp:685-953) as five
// kernels, the LM head with the greedy pick folded in, and the model engine that replays the whole
// step as one CUDA graph (src/FullModel.cpp:1096-1208 feedToken/sampleNext, without the host).
//
//   k_gemv<EMBED_NORM|NORM, BIAS>  rms_norm (+ embedding gather on layer 0) -> stacked QKV GEMV + bias
//   k_attention<FUSED>             NeoX RoPE of q and k, KV append, split-K GQA attention partials
//   k_gemv<MERGE, RESIDUAL>        merge of the attention partials -> o_proj GEMV + residual add
//   k_gemv<NORM, SWIGLU>           rms_norm -> gate and up GEMVs (one pass, two matrices) -> SwiGLU
//   k_gemv<PLAIN, RESIDUAL>        down_proj GEMV (K split across warps) + residual add
//   k_gemv<NORM, LOGITS>           final rms_norm -> LM head GEMV -> logits, argmax, next token
#include <algorithm>
#include <climits>
#include <cmath>
#include <cstddef>
#include <cstring>
#include <map>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "attention.cuh"
#include "common.cuh"

// sampler.cu: parameter check and launch of the device sampler (gate = the model's {step,
// prompt_end, total}, see k_sample).
int sample_check(const MuyoSamplerParams* p, uint32_t vocab, long long max_hist);
int sample_launch(const MuyoSamplerParams* p, float* logits, uint32_t vocab, const int32_t* history,
                  uint32_t hist_len, void* state, int32_t* token, const int32_t* gate, int32_t* tokens,
                  int max_seq, bool pdl, cudaStream_t s);
#include "gemv.cuh"

namespace muyo {
struct Pair {
    float v;
    int i;
};

// Device-resident decode control: the step counter is the position; tokens[] holds every fed and
// generated id by position (the reference's `fed`, src/FullModel.cpp:1061).
struct Control {
    int32_t step;        // position of the token being decoded
    int32_t prompt_end;  // tokens[s] for s < prompt_end are forced (prompt), later ones are generated
    int32_t total;       // tokens[] is written for positions < total
    int32_t greedy;      // the last step's raw argmax
};
static_assert(offsetof(Control, prompt_end) == 4 && offsetof(Control, total) == 8, "sampler gate layout");
}  // namespace muyo

#include "sync.cuh"
#include "decode_stream.cuh"
#include "prefill.cuh"  // after the mbarrier helpers it uses

namespace muyo {

constexpr int kGemvThreads = 256;  // 8 warps
constexpr int kGemvWarps = kGemvThreads / 32;

enum Prologue { PRO_PLAIN = 0, PRO_NORM = 1, PRO_EMBED_NORM = 2, PRO_MERGE = 3 };
enum Epilogue { EPI_BIAS = 1, EPI_RESIDUAL = 2, EPI_SWIGLU = 3, EPI_LOGITS = 4 };

// Weights of a later kernel to stream into L2 (byte ranges, 16-byte aligned, sizes multiples of 16).
struct PfSet {
    const void* p[2];
    size_t bytes[2];
    size_t per_cta[2];  // slice of each range per CTA (a multiple of 16), set at launch
};

struct GemvFused {
    // prologue
    const float* x;        // PLAIN / NORM input
    const float* norm_w;   // NORM weight
    float eps;
    const __half* embd;    // EMBED_NORM table [vocab][K]
    const int32_t* tokens;
    const Control* ctrl_ro;
    int vocab, max_seq;    // EMBED_NORM bounds
    float* x_copy;         // EMBED_NORM: CTA 0 stores the embedded row (the residual stream)
    const float* attn_part;  // MERGE: split-K attention partials [kv_heads][max_chunks][gqa][hd + 2]
    const int32_t* pos;      // MERGE: device position (keys 0 .. pos)
    int hd, gqa, max_chunks; // MERGE: partial layout
    int K;
    // matrices
    const __half* w0;
    const __half* w1;
    size_t ldw;
    int rows;
    // epilogue
    const float* bias;
    const float* res;
    float* y;
    Pair* part;         // LOGITS: per-CTA best
    int32_t* counter;   // LOGITS: arrival counter (self-resetting)
    Control* ctrl;      // LOGITS: next-token selection and step advance
    int32_t* tokens_rw;
    PfSet pf;           // weights of a later kernel: every CTA asks L2 for its slice of them
    // SW (weights in shared memory): byte offset of the weight tile in dynamic shared memory, and
    // the error word a timed-out wait for the tile sets (MUYO_ETIMEOUT on the host)
    unsigned wofs;
    int* err;
    int prefetch_all;  // non-SW path: every CTA asks L2 for all its rows before the dependency wait
};

// Stage the merged attention output (the O projection's input, K = heads * hd) from the split-K
// partials (m, l, o) of every (head, chunk): per head M = max_c m_c, w_c = exp(m_c - M) / L with
// L = sum_c l_c exp(m_c - M), then x[h * hd + d] = sum_c o_c[d] w_c. Each pass issues its loads
// together: the statistics of all heads and chunks, then four chunks of every element a thread
// owns. `scratch` holds 2 * heads * max_chunks floats.
__device__ __forceinline__ void stage_merge(const GemvFused& a, float4* xs4, float* scratch, int pos)
{
    float* xs = reinterpret_cast<float*>(xs4);
    const int K = a.K, K8 = K / 8, hd = a.hd, G = a.gqa, heads = K / hd, stride = hd + 2;
    const int tid = threadIdx.x, nt = blockDim.x;
    const int nchunks = pos >= 0 && pos < a.max_seq ? (pos + kAttnKeys) / kAttnKeys : 0;
    auto part_at = [&](int h, int c) { return a.attn_part + ((size_t)((h / G) * a.max_chunks + c) * G + h % G) * stride; };
    constexpr int E = 4;                        // elements per thread per pass
    const size_t cstride = (size_t)G * stride;  // floats between chunk c and c + 1 of one head
    const float* src[E];                        // element e's value in chunk 0
    int head[E];
    auto locate = [&](int e0) {
#pragma unroll
        for (int j = 0; j < E; ++j) {
            const int e = min(e0 + tid + j * nt, K - 1), h = e / hd;
            head[j] = h;
            src[j] = part_at(h, 0) + 2 + (e - h * hd);
        }
    };
    // The first pass's values of chunks 0..3 do not depend on the statistics: their loads go out
    // together with the statistics' loads.
    locate(0);
    float v0[E][4];
#pragma unroll
    for (int j = 0; j < E; ++j)
#pragma unroll
        for (int u = 0; u < 4; ++u)
            v0[j][u] = u < nchunks ? __ldcg(src[j] + (size_t)u * cstride) : 0.0f;
    float* mw = scratch;                   // [heads][nchunks]: m, then the normalised weight
    float* lw = scratch + heads * nchunks; // [heads][nchunks]: l
    for (int i = tid; i < heads * nchunks; i += nt) {
        const float* q = part_at(i / nchunks, i % nchunks);
        mw[i] = __ldcg(q);
        lw[i] = __ldcg(q + 1);
    }
    __syncthreads();
    for (int h = tid; h < heads; h += nt) {
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
    __syncthreads();
    for (int e0 = 0; e0 < K; e0 += E * nt) {
        if (e0 > 0)
            locate(e0);
        float o[E];
#pragma unroll
        for (int j = 0; j < E; ++j)
            o[j] = 0.0f;
        for (int c = 0; c < nchunks; c += 4) {
            float v[E][4];
#pragma unroll
            for (int j = 0; j < E; ++j)
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    v[j][u] = e0 == 0 && c == 0 ? v0[j][u]
                                                : (c + u < nchunks ? __ldcg(src[j] + (size_t)(c + u) * cstride) : 0.0f);
#pragma unroll
            for (int j = 0; j < E; ++j) {
                const float* w = mw + head[j] * nchunks;
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (c + u < nchunks)
                        o[j] = fmaf(v[j][u], w[c + u], o[j]);
            }
        }
#pragma unroll
        for (int j = 0; j < E; ++j) {
            const int e = e0 + tid + j * nt;
            if (e < K)
                xs[xs_index(e, K8)] = o[j];
        }
    }
    __syncthreads();
}

// Stage the GEMV input vector in shared memory (split layout of gemv.cuh). NORM and EMBED_NORM
// apply the numpy reference's rms_norm, x / sqrt(mean(x^2) + eps) * w (tools/reference_qwen2.py:81-82),
// in F32: the sum of squares with per-thread FMA partials and a shuffle tree.
template <int PRO>
__device__ __forceinline__ void stage_input(const GemvFused& a, float* xs, float* red, int pos = 0)
{
    // Every thread issues all loads of a pass (V float4s of x or of the embedding row, and of the
    // norm weight) before its first store, so a pass costs one memory round trip; K <= 4 * V * 256
    // takes one pass (8192 plain, 4096 normalised). K is a multiple of 8 (make_shape).
    constexpr int V = PRO == PRO_PLAIN ? 8 : 4;
    const int K = a.K, K8 = K / 8, Q = K / 4;
    float4* xs4 = reinterpret_cast<float4*>(xs);
    const int tid = threadIdx.x, nt = blockDim.x;
    if (PRO == PRO_PLAIN) {
        const float4* x4 = reinterpret_cast<const float4*>(a.x);
        for (int q0 = 0; q0 < Q; q0 += V * nt) {
            float4 v[V];
#pragma unroll
            for (int j = 0; j < V; ++j) {
                const int q = q0 + tid + j * nt;
                if (q < Q)
                    v[j] = __ldg(x4 + q);
            }
#pragma unroll
            for (int j = 0; j < V; ++j) {
                const int q = q0 + tid + j * nt;
                if (q < Q)
                    xs4[xs_slot4(q, K8)] = v[j];
            }
        }
        __syncthreads();
        return;
    }
    if (PRO == PRO_MERGE) {
        stage_merge(a, xs4, xs + K, pos);
        return;
    }
    const __half* erow = nullptr;
    if (PRO == PRO_EMBED_NORM) {
        // Ids and positions are bounded on the host; an out-of-range value read here gathers row 0
        // rather than reading outside the table.
        const int step = a.ctrl_ro->step;
        int token = step >= 0 && step < a.max_seq ? a.tokens[step] : 0;
        if (token < 0 || token >= a.vocab)
            token = 0;
        erow = a.embd + (size_t)token * K;
    }
    const float4* w4 = reinterpret_cast<const float4*>(a.norm_w);
    float4 wv[V];  // the norm weights of the first pass, loaded with the inputs
    float ss = 0.0f;
    for (int q0 = 0; q0 < Q; q0 += V * nt) {
        float4 v[V];
#pragma unroll
        for (int j = 0; j < V; ++j) {
            const int q = q0 + tid + j * nt;
            if (q < Q) {
                if (PRO == PRO_EMBED_NORM) {
                    const uint2 h = __ldg(reinterpret_cast<const uint2*>(erow) + q);
                    const float2 lo = h2_to_f2(h.x), hi = h2_to_f2(h.y);
                    v[j] = make_float4(lo.x, lo.y, hi.x, hi.y);
                } else {
                    v[j] = __ldg(reinterpret_cast<const float4*>(a.x) + q);
                }
                if (q0 == 0)
                    wv[j] = __ldg(w4 + q);
            }
        }
#pragma unroll
        for (int j = 0; j < V; ++j) {
            const int q = q0 + tid + j * nt;
            if (q < Q) {
                ss = fmaf(v[j].x, v[j].x, ss);
                ss = fmaf(v[j].y, v[j].y, ss);
                ss = fmaf(v[j].z, v[j].z, ss);
                ss = fmaf(v[j].w, v[j].w, ss);
                xs4[xs_slot4(q, K8)] = v[j];
                if (PRO == PRO_EMBED_NORM && blockIdx.x == 0)
                    reinterpret_cast<float4*>(a.x_copy)[q] = v[j];
            }
        }
    }
    ss = block_sum(ss, red);
    const float s = __fsqrt_rn(__fdiv_rn(ss, (float)K) + a.eps);
    // Each thread rescales the float4s it stored itself: x / s * w, as the numpy reference.
    for (int q0 = 0; q0 < Q; q0 += V * nt) {
#pragma unroll
        for (int j = 0; j < V; ++j) {
            const int q = q0 + tid + j * nt;
            if (q < Q) {
                const float4 w = q0 == 0 ? wv[j] : __ldg(w4 + q);
                float4& x = xs4[xs_slot4(q, K8)];
                x = make_float4(__fdiv_rn(x.x, s) * w.x, __fdiv_rn(x.y, s) * w.y, __fdiv_rn(x.z, s) * w.z,
                                __fdiv_rn(x.w, s) * w.w);
            }
        }
    }
    __syncthreads();
}

// One CTA = 8 warps = (8 / KSPLIT) row groups of ROWS rows, the K range of each row group split
// over KSPLIT warps; partial sums meet in shared memory and are added in a fixed order.
// With SW every CTA owns exactly one tile (grid == tiles) and bulk-copies the tile's weight rows
// (row stride == K, so the tile is one contiguous block per matrix) into shared memory before it
// waits for the previous kernel; it then computes from shared memory. A wait for the copies that
// exceeds kWaitLimitNs sets *a.err and skips the arithmetic.
template <int ROWS, int U, int NMAT, int KSPLIT, int PRO, int EPI, bool SW = false>
__global__ void __launch_bounds__(kGemvThreads) k_gemv(GemvFused a)
{
    extern __shared__ __align__(128) float xs[];
    __shared__ float red[32];
    __shared__ float ksum[kGemvWarps][NMAT][ROWS];
    __shared__ Pair best_sm[kGemvWarps];
    __shared__ int last_flag;
    __shared__ __align__(8) uint64_t wbar;
    constexpr int RG = kGemvWarps / KSPLIT;
    const unsigned tile_bytes = SW ? (unsigned)(RG * ROWS) * (unsigned)a.K * 2u : 0u;  // per matrix

    if (SW) {
        if (threadIdx.x == 0) {
            const int r0 = blockIdx.x * RG * ROWS, nr = min(RG * ROWS, a.rows - r0);
            const unsigned bytes = (unsigned)nr * (unsigned)a.K * 2u;
            char* wsm = reinterpret_cast<char*>(xs) + a.wofs;
            mbar_init(&wbar, 1);
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_expect_tx(&wbar, bytes * NMAT);
            bulk_g2s(wsm, a.w0 + (size_t)r0 * a.K, bytes, &wbar);
            if (NMAT > 1)
                bulk_g2s(wsm + tile_bytes, a.w1 + (size_t)r0 * a.K, bytes, &wbar);
        }
    } else if (threadIdx.x == 0) {
        // The weights do not depend on the previous kernel: start streaming this CTA's tiles into L2
        // while the previous kernel drains and the input is staged - all of them when the matrices fit
        // L2 (prefetch_all), else the first.
        const int ntl = (a.rows + RG * ROWS - 1) / (RG * ROWS);
        for (int t = blockIdx.x; t < ntl; t += gridDim.x) {
            const int r0 = t * RG * ROWS, nr = min(RG * ROWS, a.rows - r0);
            prefetch_rows_l2(a.w0, a.ldw, r0, nr);
            if (NMAT > 1)
                prefetch_rows_l2(a.w1, a.ldw, r0, nr);
            if (!a.prefetch_all)
                break;
        }
    }
    if (threadIdx.x == 0) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const size_t n = a.pf.bytes[r];
            const size_t per = a.pf.per_cta[r];
            const size_t off = (size_t)blockIdx.x * per;
            if (n > 0 && off < n) {
                const char* base = static_cast<const char*>(a.pf.p[r]) + off;
                size_t left = n - off < per ? n - off : per;
                while (left > 0) {
                    const uint32_t c = left > 65536 ? 65536u : (uint32_t)left;
                    prefetch_l2(base, c);
                    base += c;
                    left -= c;
                }
            }
        }
    }
    // MERGE: the position was written two or more launches back (by the previous step's LM head,
    // or before a launch without programmatic serialisation), so it is read before the wait.
    const int pos = PRO == PRO_MERGE ? __ldcg(a.pos) : 0;
    pdl_wait();  // the input vector and the epilogue operands come from earlier kernels
    pdl_trigger();
    stage_input<PRO>(a, xs, red, pos);  // ends with __syncthreads: the barrier's init is visible
    bool tile_ok = true;
    if (SW) {
        tile_ok = mbar_try_wait(&wbar, 0);
        if (!tile_ok) {
            const unsigned long long t0 = now_ns();
            while (!(tile_ok = mbar_try_wait(&wbar, 0)) && now_ns() - t0 <= kWaitLimitNs) {
            }
            if (!tile_ok) {
                atomicMax(a.err, 4);
                // the copies may still be in flight: give them one more bounded wait before exit
                const unsigned long long t1 = now_ns();
                while (!mbar_try_wait(&wbar, 0) && now_ns() - t1 <= kWaitLimitNs) {
                }
            }
        }
    }

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int rg = warp / KSPLIT, ks = warp % KSPLIT;
    const int K8 = a.K / 8;
    const int c_begin = (int)((long long)K8 * ks / KSPLIT), c_end = (int)((long long)K8 * (ks + 1) / KSPLIT);
    const int ntiles = (a.rows + RG * ROWS - 1) / (RG * ROWS);
    GemvArgs<ROWS, U, NMAT> ga;
    ga.w[0] = a.w0;
    if (NMAT > 1)
        ga.w[NMAT - 1] = a.w1;
    ga.ldw = a.ldw;
    float bv = -INFINITY;
    int bi = INT_MAX;

    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const int row0 = (tile * RG + rg) * ROWS;
        const int nvalid = min(ROWS, a.rows - row0);
        if (!SW && !a.prefetch_all && threadIdx.x == 0 && tile + (int)gridDim.x < ntiles) {  // the next tile, to L2
            const int r1 = (tile + gridDim.x) * RG * ROWS, nr = min(RG * ROWS, a.rows - r1);
            prefetch_rows_l2(a.w0, a.ldw, r1, nr);
            if (NMAT > 1)
                prefetch_rows_l2(a.w1, a.ldw, r1, nr);
        }
        // The epilogue operand of row row0 + lane (bias or residual), loaded before the weights.
        float epi_op = 0.0f;
        if ((EPI == EPI_BIAS || EPI == EPI_RESIDUAL) && ks == 0 && lane < ROWS && lane < nvalid)
            epi_op = EPI == EPI_BIAS ? a.bias[row0 + lane] : a.res[row0 + lane];
        float acc[NMAT][ROWS];
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
            for (int r = 0; r < ROWS; ++r)
                acc[m][r] = 0.0f;
        if (nvalid > 0 && tile_ok) {
            if (SW) {
                unsigned wsm[NMAT];
                const unsigned w0s = (unsigned)__cvta_generic_to_shared(reinterpret_cast<char*>(xs) + a.wofs);
#pragma unroll
                for (int m = 0; m < NMAT; ++m)
                    wsm[m] = w0s + (unsigned)m * tile_bytes;
                warp_gemv_f16_smem<ROWS, U, NMAT>(wsm, (unsigned)a.K * 2u, rg * ROWS, nvalid, xs, K8, c_begin, c_end,
                                                  lane, acc);
            } else {
                warp_gemv_f16_range<ROWS, U, NMAT>(ga, row0, nvalid, xs, K8, c_begin, c_end, lane, acc);
            }
            warp_reduce_acc<ROWS, NMAT>(acc);
        }
        if (KSPLIT > 1) {
            if (lane == 0) {
#pragma unroll
                for (int m = 0; m < NMAT; ++m)
#pragma unroll
                    for (int r = 0; r < ROWS; ++r)
                        ksum[warp][m][r] = acc[m][r];
            }
            __syncthreads();
            if (ks == 0) {  // every lane: the epilogue of row r runs in lane r
#pragma unroll
                for (int m = 0; m < NMAT; ++m)
#pragma unroll
                    for (int r = 0; r < ROWS; ++r) {
                        float t = ksum[warp][m][r];
#pragma unroll
                        for (int j = 1; j < KSPLIT; ++j)
                            t += ksum[warp + j][m][r];
                        acc[m][r] = t;
                    }
            }
            __syncthreads();
        }
        if (EPI == EPI_LOGITS) {
            if (ks == 0 && lane == 0 && nvalid > 0) {
#pragma unroll
                for (int r = 0; r < ROWS; ++r) {
                    if (r >= nvalid)
                        break;
                    const int row = row0 + r;
                    const float v = acc[0][r];
                    a.y[row] = v;
                    if (pair_better(v, row, bv, bi))
                        bv = v, bi = row;
                }
            }
        } else if (ks == 0 && lane < ROWS && lane < nvalid) {
            // After the butterfly every lane holds every row's sum: lane r finishes row r, whose
            // epilogue operand it loaded itself.
            float s0 = acc[0][0], s1 = acc[NMAT - 1][0];
#pragma unroll
            for (int r = 1; r < ROWS; ++r)
                if (lane == r)
                    s0 = acc[0][r], s1 = acc[NMAT - 1][r];
            const int row = row0 + lane;
            if (EPI == EPI_BIAS)
                a.y[row] = s0 + epi_op;
            else if (EPI == EPI_RESIDUAL)
                a.y[row] = epi_op + s0;
            else  // EPI_SWIGLU
                a.y[row] = silu_mul(s0, s1);
        }
    }

    if (EPI != EPI_LOGITS)
        return;
    // Greedy pick (src/Sampler.cpp:32-43, first index of the maximum) across the grid: CTA best,
    // then the last CTA to arrive reduces all of them and advances the decode control block.
    if (lane == 0)
        best_sm[warp] = Pair{bv, bi};
    __syncthreads();
    if (warp == 0) {
        Pair p = lane < kGemvWarps ? best_sm[lane] : Pair{-INFINITY, INT_MAX};
        warp_argmax(p.v, p.i);
        if (lane == 0) {
            a.part[blockIdx.x] = p;
            __threadfence();
            last_flag = atomicAdd(a.counter, 1) == (int)gridDim.x - 1;
        }
    }
    __syncthreads();
    if (!last_flag)
        return;
    __threadfence();
    if (warp == 0) {
        float v = -INFINITY;
        int i = INT_MAX;
        for (int k = lane; k < (int)gridDim.x; k += 32) {
            const Pair q = a.part[k];
            if (pair_better(q.v, q.i, v, i))
                v = q.v, i = q.i;
        }
        warp_argmax(v, i);
        if (lane == 0) {
            const int greedy = i == INT_MAX ? 0 : i;
            Control* c = a.ctrl;
            const int s = c->step;
            if (s + 1 < c->total && s + 1 < a.max_seq) {
                const int next = s + 1 < c->prompt_end ? a.tokens_rw[s + 1] : greedy;
                a.tokens_rw[s + 1] = next;
            }
            c->greedy = greedy;
            c->step = s + 1;
            *a.counter = 0;
        }
    }
}

// Each CTA of a grid of `grid` CTAs prefetches one slice (a multiple of 16 bytes) of each range.
static void set_prefetch_slices(PfSet& pf, int grid)
{
    for (int r = 0; r < 2; ++r)
        pf.per_cta[r] = (pf.bytes[r] / (size_t)grid + 16) / 16 * 16;
}

// Every kernel of the decode step asks for the largest shared-memory carveout: the L1/shared split
// is set per SM, so a kernel that starts early (programmatic launch) can only be placed on SMs whose
// split already leaves it room, and a uniform split lets consecutive kernels share SMs.
template <typename Kernel>
static cudaError_t max_shared_carveout(Kernel k)
{
    return cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
}

// CTAs of kernel k (block threads, smem bytes) resident on the whole device at once.
template <typename Kernel>
static int resident_ctas(Kernel k, int threads, size_t smem)
{
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, threads, smem) != cudaSuccess || per_sm < 1)
        per_sm = 1;
    return per_sm * sm_count();
}

// The grid is capped at the CTAs resident at once: CTAs stride over the tiles, so a tile beyond the
// first wave reuses an already staged input instead of waiting for a second wave to start.
// With an error word (a.err) and row stride == K, the weights-in-shared-memory variant (ROWS_SW
// rows per warp, U_SW chunks in flight) is used when one tile per CTA fits the device at once.
template <int ROWS, int U, int NMAT, int KSPLIT, int PRO, int EPI, int ROWS_SW = ROWS, int U_SW = U>
static int launch_gemv(const GemvFused& a, int max_ctas, cudaStream_t s, bool pdl)
{
    constexpr int RG = kGemvWarps / KSPLIT;
    const int ntiles = (a.rows + RG * ROWS - 1) / (RG * ROWS);
    size_t smem = (size_t)a.K * sizeof(float);
    if (PRO == PRO_MERGE)
        smem += 2 * sizeof(float) * (size_t)(a.K / a.hd) * a.max_chunks;  // merge statistics
    if constexpr (EPI != EPI_LOGITS) {
      if (a.err && a.ldw == (size_t)a.K) {
        const int ntiles_sw = (a.rows + RG * ROWS_SW - 1) / (RG * ROWS_SW);
        const size_t wofs = (smem + 127) / 128 * 128;
        const size_t smem_sw = wofs + (size_t)NMAT * RG * ROWS_SW * a.K * 2;
        auto ksw = k_gemv<ROWS_SW, U_SW, NMAT, KSPLIT, PRO, EPI, true>;
        MUYO_CUDA_TRY(max_shared_carveout(ksw));
        if (smem_sw <= 200 * 1024) {
            if (smem_sw > 48 * 1024)
                MUYO_CUDA_TRY(cudaFuncSetAttribute(ksw, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_sw));
            if (resident_ctas(ksw, kGemvThreads, smem_sw) >= ntiles_sw) {
                GemvFused b = a;
                b.wofs = (unsigned)wofs;
                set_prefetch_slices(b.pf, ntiles_sw);
                MUYO_CUDA_TRY(launch_kernel(ksw, dim3(ntiles_sw), dim3(kGemvThreads), smem_sw, s, pdl, b));
                MUYO_LAUNCH_CHECK();
                return MUYO_OK;
            }
        }
      }
    }
    auto k = k_gemv<ROWS, U, NMAT, KSPLIT, PRO, EPI>;
    MUYO_CUDA_TRY(max_shared_carveout(k));
    if (smem > 48 * 1024)
        MUYO_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int grid = ntiles < max_ctas ? ntiles : max_ctas;
    GemvFused b = a;
    b.prefetch_all = (size_t)a.rows * a.ldw * 2 * NMAT <= (64ull << 20) ? 1 : 0;
    const int resident = resident_ctas(k, kGemvThreads, smem);
    if (grid > resident)
        grid = resident;
    set_prefetch_slices(b.pf, grid);
    MUYO_CUDA_TRY(launch_kernel(k, dim3(grid), dim3(kGemvThreads), smem, s, pdl, b));
    MUYO_LAUNCH_CHECK();
    return MUYO_OK;
}

// ---- shapes ------------------------------------------------------------------------------------------

struct Shape {
    int layers, hidden, ffn, heads, kv_heads, vocab, max_seq, head_dim, q_dim, kv_dim, qkv_rows, gqa;
    float eps, rope_base;
    bool kv_f16;
    int max_chunks;
    const double* rope_cs;  // optional device (cos, sin) table [max_seq][head_dim] (the model's)
};

static int make_shape(const MuyoQwen2Config* c, Shape& s, bool need_vocab)
{
    MUYO_REQUIRE(c, "config is null");
    MUYO_REQUIRE(c->hidden > 0 && c->heads > 0 && c->kv_heads > 0 && c->ffn > 0 && c->max_seq > 0,
                 "config: hidden, heads, kv_heads, ffn and max_seq must be positive");
    MUYO_REQUIRE(c->hidden % c->heads == 0, "config: hidden %u not divisible by heads %u", c->hidden, c->heads);
    MUYO_REQUIRE(c->heads % c->kv_heads == 0, "config: heads %u not divisible by kv_heads %u", c->heads, c->kv_heads);
    s.layers = (int)c->layers;
    s.hidden = (int)c->hidden;
    s.ffn = (int)c->ffn;
    s.heads = (int)c->heads;
    s.kv_heads = (int)c->kv_heads;
    s.vocab = (int)c->vocab;
    s.max_seq = (int)c->max_seq;
    s.head_dim = s.hidden / s.heads;
    s.q_dim = s.heads * s.head_dim;
    s.kv_dim = s.kv_heads * s.head_dim;
    s.qkv_rows = s.q_dim + 2 * s.kv_dim;
    s.gqa = s.heads / s.kv_heads;
    s.eps = c->rms_eps;
    s.rope_base = c->rope_base;
    MUYO_REQUIRE(c->kv_dtype == MUYO_KV_F32 || c->kv_dtype == MUYO_KV_F16, "config: kv_dtype %u", c->kv_dtype);
    s.kv_f16 = c->kv_dtype == MUYO_KV_F16;
    MUYO_REQUIRE(s.head_dim == 16 || s.head_dim == 32 || s.head_dim == 64 || s.head_dim == 128,
                 "config: head_dim %d not supported by the fused step (16, 32, 64, 128)", s.head_dim);
    MUYO_REQUIRE(s.gqa <= kAttnMaxGroup, "config: %d query heads per KV head exceed %d", s.gqa, kAttnMaxGroup);
    MUYO_REQUIRE(s.hidden % 8 == 0 && s.ffn % 8 == 0, "config: hidden and ffn must be multiples of 8");
    MUYO_REQUIRE(s.hidden <= 16384 && s.ffn <= 56 * 1024, "config: hidden/ffn too large for the staged input");
    MUYO_REQUIRE(!need_vocab || c->vocab > 0, "config: vocab must be positive");
    MUYO_REQUIRE(s.rope_base > 0.0f && s.eps >= 0.0f, "config: rope_base must be > 0 and rms_eps >= 0");
    s.max_chunks = (s.max_seq + kAttnKeys - 1) / kAttnKeys;
    MUYO_REQUIRE(sizeof(float) * ((size_t)s.q_dim + 2ull * s.heads * s.max_chunks) <= 200 * 1024,
                 "config: heads x max_seq too large for the attention merge staged in shared memory");
    return MUYO_OK;
}

// Scratch of one layer step: counters first (must start at zero; the kernels leave them zero).
struct LayerScratch {
    int32_t* counters;  // [kv_heads]
    float* qkv;         // [qkv_rows]
    float* attn;        // [q_dim]
    float* h1;          // [hidden]
    float* act;         // [ffn]
    float* part;        // attention partials
};

static size_t align256(size_t n) { return (n + 255) / 256 * 256; }

static size_t part_floats(const Shape& s) { return (size_t)s.kv_heads * s.max_chunks * s.gqa * (s.head_dim + 2); }

static size_t layer_scratch_bytes(const Shape& s)
{
    return align256(sizeof(int32_t) * (size_t)s.kv_heads) + align256(sizeof(float) * s.qkv_rows) +
           align256(sizeof(float) * s.q_dim) + align256(sizeof(float) * s.hidden) + align256(sizeof(float) * s.ffn) +
           align256(sizeof(float) * part_floats(s));
}

static LayerScratch carve_layer_scratch(const Shape& s, void* base)
{
    char* p = static_cast<char*>(base);
    LayerScratch w;
    w.counters = reinterpret_cast<int32_t*>(p);
    p += align256(sizeof(int32_t) * (size_t)s.kv_heads);
    w.qkv = reinterpret_cast<float*>(p);
    p += align256(sizeof(float) * s.qkv_rows);
    w.attn = reinterpret_cast<float*>(p);
    p += align256(sizeof(float) * s.q_dim);
    w.h1 = reinterpret_cast<float*>(p);
    p += align256(sizeof(float) * s.hidden);
    w.act = reinterpret_cast<float*>(p);
    p += align256(sizeof(float) * s.ffn);
    w.part = reinterpret_cast<float*>(p);
    return w;
}

struct LayerPtrs {
    const float* attn_norm;
    const __half* wqkv;
    const float* bqkv;
    const __half* wo;
    const float* ffn_norm;
    const __half* wgate;
    const __half* wup;
    const __half* wdown;
};

// Where the attention chunks' partials are merged. Every CTA of the O projection re-merges all of them
// while staging its input: cheap while the partial set is small (0.5B: 118 KB at 2048 positions),
// not for wide models with long caches (7B-class: 532 KB per CTA). Above this size the last CTA of
// each KV head merges its group's partials and writes the attention output instead.
constexpr size_t kMergeInOBytes = 128 * 1024;

static bool merge_in_o(const Shape& s)
{
    return sizeof(float) * (size_t)s.heads * s.max_chunks * (s.head_dim + 2) <= kMergeInOBytes;
}

template <typename KV, int HD>
static int launch_attention_fused(const Shape& s, const float* qkv, void* kc, void* vc, const int32_t* pos,
                                  float* out, float* part, int32_t* counters, cudaStream_t st, bool pdl)
{
    AttnDev p{s.heads, s.kv_heads, s.gqa, s.max_seq, 0, 1.0f / sqrtf((float)s.head_dim), (double)s.rope_base,
              s.max_chunks, s.rope_cs};
    const size_t smem = (size_t)attn_smem_floats(HD, s.gqa) * sizeof(float);
    // merge_in_o: every chunk writes its partial and the O projection merges them while staging its
    // input; else the last CTA of each KV head merges into `out` (a single chunk writes it directly).
    const bool in_o = merge_in_o(s);
    auto k = in_o ? k_attention<KV, HD, true, false> : k_attention<KV, HD, true, true>;
    MUYO_CUDA_TRY(max_shared_carveout(k));
    if (smem > 48 * 1024)
        MUYO_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    MUYO_CUDA_TRY(launch_kernel(k, dim3(s.kv_heads, s.max_chunks), dim3(kAttnThreads), smem, st, pdl, p, qkv,
                                static_cast<KV*>(kc), static_cast<KV*>(vc), pos, in_o ? nullptr : out, part,
                                counters));
    MUYO_LAUNCH_CHECK();
    return MUYO_OK;
}

static int attention_fused(const Shape& s, const float* qkv, void* kc, void* vc, const int32_t* pos, float* out,
                           float* part, int32_t* counters, cudaStream_t st, bool pdl)
{
    if (s.kv_f16) {
        switch (s.head_dim) {
            case 16: return launch_attention_fused<__half, 16>(s, qkv, kc, vc, pos, out, part, counters, st, pdl);
            case 32: return launch_attention_fused<__half, 32>(s, qkv, kc, vc, pos, out, part, counters, st, pdl);
            case 64: return launch_attention_fused<__half, 64>(s, qkv, kc, vc, pos, out, part, counters, st, pdl);
            default: return launch_attention_fused<__half, 128>(s, qkv, kc, vc, pos, out, part, counters, st, pdl);
        }
    }
    switch (s.head_dim) {
        case 16: return launch_attention_fused<float, 16>(s, qkv, kc, vc, pos, out, part, counters, st, pdl);
        case 32: return launch_attention_fused<float, 32>(s, qkv, kc, vc, pos, out, part, counters, st, pdl);
        case 64: return launch_attention_fused<float, 64>(s, qkv, kc, vc, pos, out, part, counters, st, pdl);
        default: return launch_attention_fused<float, 128>(s, qkv, kc, vc, pos, out, part, counters, st, pdl);
    }
}

// One decoder layer: x_in (or the embedding of tokens[ctrl->step] when embed != nullptr) -> x_out.
static int layer_forward(const Shape& s, const LayerPtrs& w, void* kc, void* vc, const int32_t* pos,
                         const float* x_in, float* x_out, const LayerScratch& ws, const __half* embd,
                         const int32_t* tokens, const Control* ctrl, float* embed_out, cudaStream_t st, bool pdl,
                         const PfSet* pf = nullptr, int* err = nullptr)
{
    const int sms = sm_count();
    int rc;
    GemvFused a{};
    a.eps = s.eps;
    a.ldw = s.hidden;
    // 1. rms_norm -> QKV GEMV + bias
    a.x = x_in;
    a.norm_w = w.attn_norm;
    a.K = s.hidden;
    a.w0 = w.wqkv;
    a.rows = s.qkv_rows;
    a.bias = w.bqkv;
    a.y = ws.qkv;
    a.err = err;
    if (pf)
        a.pf = pf[0];
    if (embd) {
        a.embd = embd;
        a.tokens = tokens;
        a.ctrl_ro = ctrl;
        a.vocab = s.vocab;
        a.max_seq = s.max_seq;
        a.x_copy = embed_out;
        rc = launch_gemv<1, 8, 1, 1, PRO_EMBED_NORM, EPI_BIAS, 2, 4>(a, sms * 8, st, pdl);
    } else {
        rc = launch_gemv<1, 8, 1, 1, PRO_NORM, EPI_BIAS, 2, 4>(a, sms * 8, st, pdl);
    }
    if (rc)
        return rc;
    const float* residual = embd ? embed_out : x_in;
    // 2. rope + KV append + attention
    rc = attention_fused(s, ws.qkv, kc, vc, pos, ws.attn, ws.part, ws.counters, st, pdl);
    if (rc)
        return rc;
    // 3. merge of the attention partials (or the merged output) -> o_proj + residual
    GemvFused o{};
    o.attn_part = ws.part;
    o.pos = pos;
    o.hd = s.head_dim;
    o.gqa = s.gqa;
    o.max_chunks = s.max_chunks;
    o.max_seq = s.max_seq;
    o.K = s.q_dim;
    o.w0 = w.wo;
    o.ldw = s.q_dim;
    o.rows = s.hidden;
    o.res = residual;
    o.y = ws.h1;
    o.err = err;
    if (pf)
        o.pf = pf[1];
    if (merge_in_o(s)) {
        // Every CTA merges all partials while staging its input: narrow models take fewer, larger
        // CTAs (16 rows each, 56 for the 0.5B O projection; ~1% of the step against 112 CTAs).
        if (s.hidden >= 2048)
            rc = launch_gemv<1, 4, 1, 2, PRO_MERGE, EPI_RESIDUAL, 2, 4>(o, sms * 8, st, pdl);
        else
            rc = launch_gemv<1, 4, 1, 1, PRO_MERGE, EPI_RESIDUAL, 2, 2>(o, sms * 8, st, pdl);
    } else {
        o.x = ws.attn;
        rc = launch_gemv<1, 4, 1, 2, PRO_PLAIN, EPI_RESIDUAL, 2, 4>(o, sms * 8, st, pdl);
    }
    if (rc)
        return rc;
    // 4. rms_norm -> gate, up -> SwiGLU
    GemvFused g{};
    g.x = ws.h1;
    g.norm_w = w.ffn_norm;
    g.eps = s.eps;
    g.K = s.hidden;
    g.w0 = w.wgate;
    g.w1 = w.wup;
    g.ldw = s.hidden;
    g.rows = s.ffn;
    g.y = ws.act;
    g.err = err;
    if (pf)
        g.pf = pf[2];
    // Wide rows (7B-class) split each row's K range over two warps, which doubles the CTAs' rows in
    // flight (111 against 118 us per 7B-class layer); narrow ones keep whole rows per warp, with two
    // rows per warp in the shared-memory tiles (304 CTAs for the 0.5B FFN).
    if (s.hidden >= 2048)
        rc = launch_gemv<1, 8, 2, 2, PRO_NORM, EPI_SWIGLU, 3, 2>(g, sms * 8, st, pdl);
    else
        rc = launch_gemv<1, 4, 2, 1, PRO_NORM, EPI_SWIGLU, 2, 2>(g, sms * 8, st, pdl);
    if (rc)
        return rc;
    // 5. down_proj + residual
    GemvFused d{};
    d.x = ws.act;
    d.K = s.ffn;
    d.w0 = w.wdown;
    d.ldw = s.ffn;
    d.rows = s.hidden;
    d.res = ws.h1;
    d.y = x_out;
    d.err = err;
    if (pf)
        d.pf = pf[3];
    // Narrow models: 8 rows per CTA, each row's K range over two warps (112 CTAs for the 0.5B down
    // projection, 3% of the step against 224 CTAs of 4 rows); wide ones split K over four warps.
    if (s.hidden >= 2048)
        return launch_gemv<1, 8, 1, 4, PRO_PLAIN, EPI_RESIDUAL, 2, 4>(d, sms * 8, st, pdl);
    return launch_gemv<1, 8, 1, 2, PRO_PLAIN, EPI_RESIDUAL, 2, 4>(d, sms * 8, st, pdl);
}

// ---- model ------------------------------------------------------------------------------------------

struct TensorSlot {
    size_t offset;  // bytes into the arena
    size_t bytes;
    bool f16;
    bool set;
};

}  // namespace muyo

struct MuyoModel {
    muyo::Shape s;
    int device = 0;
    char* arena = nullptr;  // weights
    size_t arena_bytes = 0;
    std::map<std::string, muyo::TensorSlot> slots;
    bool tied_output = true;
    void* kc = nullptr;
    void* vc = nullptr;
    size_t kv_layer_bytes = 0;
    char* scratch = nullptr;  // activations, partials, control (zeroed at create)
    muyo::LayerScratch ls{};
    float* h = nullptr;
    float* logits = nullptr;
    muyo::Pair* lm_part = nullptr;
    int32_t* lm_counter = nullptr;
    muyo::Control* ctrl = nullptr;
    int32_t* tokens = nullptr;
    int lm_grid = 0;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    // kGraphSteps consecutive steps in one graph: inside it each step's first kernel starts under the
    // previous step's LM head (programmatic launch), which separate graph launches do not allow
    cudaGraph_t graph_n = nullptr;
    cudaGraphExec_t exec_n = nullptr;
    cudaStream_t cap_stream = nullptr;
    int32_t* pinned = nullptr;  // host staging for prompt/output (generate/step synchronise before reuse)
    size_t pinned_ints = 0;
    int32_t host_pos = 0;
    bool finalized = false;
    int engine = 1;                 // 0: streaming persistent kernel, 1: CUDA graph of per-phase kernels (default)
    bool pdl = true;                // graph engine: kernels launch early and prefetch their weights
    bool prefetch_ahead = true;     // graph engine: each GEMV streams a later kernel's weights into L2
    bool sw = true;                 // graph engine: per-layer GEMVs bulk-copy their weight tile to shared memory
    bool sampling = false;          // graph engine: a device sampler node follows the LM head
    MuyoSamplerParams sp{};         // its parameters (baked into the recorded graph)
    void* rng = nullptr;            // its mt19937_64 state, followed by the last sampled id (int32)
    bool prefill = false;           // generate: the prompt's positions but the last in one batched pass
    int pf_tc = 2;                  // prefill projections: 0 mma.sync, 1 tcgen05, 2 per GEMM (option "prefill_tc")
    std::vector<CUtensorMap> pf_maps;  // tcgen05 prefill: 5 weight maps per layer, then the activation halves
    char* pf_buf = nullptr;         // batched-prefill activations for pf_cap positions
    int pf_cap = 512;               // positions per prefill pass (option "prefill_positions")
    float *pf_x = nullptr, *pf_qkv = nullptr, *pf_q = nullptr, *pf_att = nullptr, *pf_gu = nullptr;
    float* pf_part = nullptr;  // split-K partial sums
    size_t pf_part_floats = 0;
    __half *pf_hi = nullptr, *pf_lo = nullptr;
    double* rope_cs = nullptr;      // [max_seq][head_dim] cos/sin table (float64)
    int* err = nullptr;             // error word of the bounded device waits
    // streaming persistent engine (decode_stream.cuh)
    muyo::SLayer* d_slayers = nullptr;
    unsigned long long* ll = nullptr;  // tagged hand-off words: per-layer blocks, then the greedy pairs
    int* abort_g = nullptr;         // the launch's abort word
    muyo::SArgs sa{};               // everything but the per-launch fields
    int s_smem = 0, s_grid = 0;
    bool s_ok = false;              // the shapes fit the streaming kernel
    std::string s_why;              // why not, when they do not
    unsigned s_tag = 1;             // tag of the next step (never 0)
};

namespace muyo {

static const __half* W(const MuyoModel* m, const std::string& name)
{
    return reinterpret_cast<const __half*>(m->arena + m->slots.at(name).offset);
}
static const float* F(const MuyoModel* m, const std::string& name)
{
    return reinterpret_cast<const float*>(m->arena + m->slots.at(name).offset);
}

static LayerPtrs layer_ptrs(const MuyoModel* m, int l)
{
    const std::string p = "blk." + std::to_string(l) + ".";
    LayerPtrs w;
    w.attn_norm = F(m, p + "attn_norm.weight");
    w.wqkv = W(m, p + "attn_qkv.weight");
    w.bqkv = F(m, p + "attn_qkv.bias");
    w.wo = W(m, p + "attn_output.weight");
    w.ffn_norm = F(m, p + "ffn_norm.weight");
    w.wgate = W(m, p + "ffn_gate.weight");
    w.wup = W(m, p + "ffn_up.weight");
    w.wdown = W(m, p + "ffn_down.weight");
    return w;
}

static int32_t* sampled_id(MuyoModel* m)
{
    return reinterpret_cast<int32_t*>(static_cast<char*>(m->rng) + (muyo_sampler_state_bytes() + 15) / 16 * 16);
}

// Records one whole decode step on stream st (5 kernels per layer + the LM head, + the sampler).
static int record_step(MuyoModel* m, cudaStream_t st)
{
    const Shape& s = m->s;
    const int32_t* pos = &m->ctrl->step;
    int rc;
    // The GEMV kernels of a step in launch order (QKV, O, gate/up, down per layer, then the LM head),
    // each with its weights. Kernel k asks L2 for the weights of kernel k + 2 (the step is replayed,
    // so the last kernels fetch the first ones of the next step), except for the LM head's, which
    // are larger than L2 and are streamed by the LM head itself.
    std::vector<PfSet> mats;
    const size_t hid = s.hidden, ffn = s.ffn;
    for (int l = 0; l < s.layers; ++l) {
        const LayerPtrs w = layer_ptrs(m, l);
        mats.push_back(PfSet{{w.wqkv, nullptr}, {(size_t)s.qkv_rows * hid * 2, 0}});
        mats.push_back(PfSet{{w.wo, nullptr}, {hid * (size_t)s.q_dim * 2, 0}});
        mats.push_back(PfSet{{w.wgate, w.wup}, {ffn * hid * 2, ffn * hid * 2}});
        mats.push_back(PfSet{{w.wdown, nullptr}, {hid * ffn * 2, 0}});
    }
    const size_t n_mats = mats.size() + 1;  // + the LM head
    std::vector<PfSet> plan(n_mats, PfSet{{nullptr, nullptr}, {0, 0}});
    if (m->prefetch_ahead)
        for (size_t k = 0; k < n_mats; ++k) {
            const size_t t = (k + 2) % n_mats;
            if (t < mats.size())
                plan[k] = mats[t];
        }
    for (int l = 0; l < s.layers; ++l) {
        const LayerPtrs w = layer_ptrs(m, l);
        char* kc = static_cast<char*>(m->kc) + m->kv_layer_bytes * l;
        char* vc = static_cast<char*>(m->vc) + m->kv_layer_bytes * l;
        if (l == 0)
            rc = layer_forward(s, w, kc, vc, pos, nullptr, m->h, m->ls, W(m, "token_embd.weight"), m->tokens,
                               m->ctrl, m->ls.h1 /*embedding row lands in h1 first*/, st, m->pdl, &plan[4 * l],
                               m->sw ? m->err : nullptr);
        else
            rc = layer_forward(s, w, kc, vc, pos, m->h, m->h, m->ls, nullptr, nullptr, nullptr, nullptr, st, m->pdl,
                               &plan[4 * l], m->sw ? m->err : nullptr);
        if (rc)
            return rc;
    }
    GemvFused a{};
    a.x = m->h;
    a.norm_w = F(m, "output_norm.weight");
    a.eps = s.eps;
    a.K = s.hidden;
    a.w0 = W(m, m->tied_output ? "token_embd.weight" : "output.weight");
    a.ldw = s.hidden;
    a.rows = s.vocab;
    a.y = m->logits;
    a.part = m->lm_part;
    a.counter = m->lm_counter;
    a.ctrl = m->ctrl;
    a.tokens_rw = m->tokens;
    a.max_seq = s.max_seq;
    a.pf = plan[n_mats - 1];
    rc = launch_gemv<2, 4, 1, 1, PRO_NORM, EPI_LOGITS>(a, m->lm_grid, st, m->pdl);
    if (rc || !m->sampling)
        return rc;
    // Non-greedy decoding: the sampler replaces the LM head's pick at generated positions
    // (Sampler::Sample on the logits with every cached id as history, src/FullModel.cpp:1111-1116).
    return sample_launch(&m->sp, m->logits, (uint32_t)s.vocab, nullptr, 0, m->rng, sampled_id(m), &m->ctrl->step,
                         m->tokens, s.max_seq, false, st);
}

// ---- streaming persistent engine -------------------------------------------------------------------

constexpr int kSmemLimit = 227 * 1024;

static size_t round16w(size_t n) { return (n + 15) / 16 * 16; }  // words, keeping 128-byte alignment
static int round128i(size_t n) { return (int)((n + 127) / 128 * 128); }

// Shared-memory and hand-off-buffer plan of the streaming kernel (decode_stream.cuh). Sets m->s_ok, or
// m->s_why when the shapes do not fit it (the graph engine then runs them).
static int stream_plan(MuyoModel* m)
{
    const Shape& s = m->s;
    m->s_ok = false;
    m->s_why.clear();
    const int hd = s.head_dim;
    if (s.heads > 64) {
        m->s_why = "more than 64 query heads";
        return MUYO_OK;
    }
    const int xs_floats = (std::max(std::max(s.hidden, s.q_dim), s.ffn) + 3) / 4 * 4;
    // The merge's staged partials or the attention scratch follow the first q_dim floats of xs.
    const size_t merge_floats = (size_t)s.heads * kSJmax * (hd + 3);
    const size_t attn_floats = 5 * (size_t)hd + 2 * kSKeys + 4 + 512;
    const size_t work_floats = std::max((size_t)xs_floats, (size_t)(s.q_dim + 3) / 4 * 4 + std::max(merge_floats, attn_floats));
    const int off_work = 0;  // relative to the end of the ring
    const int off_hraw = off_work + round128i(work_floats * sizeof(float));
    const int off_h1raw = off_hraw + round128i((size_t)s.hidden * sizeof(float));
    const int off_misc = off_h1raw + round128i((size_t)s.hidden * sizeof(float));
    const int fixed = off_misc + round128i(s_misc_bytes());
    // The largest piece of any phase (whole rows, at least one).
    struct Ph { int K, nmat, M; bool head; } phs[5] = {{s.hidden, 1, s.qkv_rows, false}, {s.q_dim, 1, s.hidden, false},
                                                      {s.hidden, 2, s.ffn, false}, {s.ffn, 1, s.hidden, false},
                                                      {s.hidden, 1, s.vocab, true}};
    size_t max_piece = 0;
    for (const Ph& p : phs)
        max_piece = std::max(max_piece, (size_t)round128i((size_t)s_rows_per_piece(p.K, p.nmat, p.head) * p.K * 2 * p.nmat));
    const int ring = (kSmemLimit - fixed) / 128 * 128;
    if (ring < (int)(2 * max_piece) || ring < 2 * 16384) {
        m->s_why = "the shapes leave too little shared memory for the weight ring";
        return MUYO_OK;
    }
    SArgs& a = m->sa;
    a = SArgs{};
    a.L = s.layers;
    a.H = s.hidden;
    a.F = s.ffn;
    a.V = s.vocab;
    a.QKV = s.qkv_rows;
    a.QD = s.q_dim;
    a.KVD = s.kv_dim;
    a.heads = s.heads;
    a.kv_heads = s.kv_heads;
    a.gqa = s.gqa;
    a.max_seq = s.max_seq;
    a.eps = s.eps;
    a.scale = 1.0f / sqrtf((float)hd);
    a.ring_bytes = ring;
    a.off_work = ring + off_work;
    a.off_hraw = ring + off_hraw;
    a.off_h1raw = ring + off_h1raw;
    a.off_misc = ring + off_misc;
    a.xs_floats = xs_floats;
    m->s_smem = ring + fixed;
    // Tagged words: per layer qkv, attention partials, h1, SwiGLU output, layer output; then the
    // double-buffered greedy pairs of every CTA.
    size_t w = 0;
    a.o_qkv = (int)w;
    w += round16w(s.qkv_rows);
    a.o_part = (int)w;
    w += round16w((size_t)s.heads * kSJmax * (hd + 2));
    a.o_h1 = (int)w;
    w += round16w(s.hidden);
    a.o_act = (int)w;
    w += round16w(s.ffn);
    a.o_hout = (int)w;
    w += round16w(s.hidden);
    a.ll_layer = (long long)w;
    m->s_ok = true;
    return MUYO_OK;
}

// Device buffers and the cooperative-launch check of the streaming kernel (once per model).
template <typename KV, int HD>
static int stream_setup_t(MuyoModel* m)
{
    auto k = k_decode_stream<KV, HD>;
    MUYO_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, m->s_smem));
    int per_sm = 0;
    MUYO_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kSThreads, m->s_smem));
    if (per_sm < 1) {
        m->s_ok = false;
        m->s_why = "the streaming kernel does not fit on an SM";
        return MUYO_OK;
    }
    m->s_grid = sm_count();
    return MUYO_OK;
}

#define MUYO_STREAM_DISPATCH(FN, ...)                                                        \
    do {                                                                                     \
        const Shape& s_ = m->s;                                                              \
        if (s_.kv_f16) {                                                                     \
            switch (s_.head_dim) {                                                           \
                case 16: return FN<__half, 16>(__VA_ARGS__);                                 \
                case 32: return FN<__half, 32>(__VA_ARGS__);                                 \
                case 64: return FN<__half, 64>(__VA_ARGS__);                                 \
                default: return FN<__half, 128>(__VA_ARGS__);                                \
            }                                                                                \
        }                                                                                    \
        switch (s_.head_dim) {                                                               \
            case 16: return FN<float, 16>(__VA_ARGS__);                                      \
            case 32: return FN<float, 32>(__VA_ARGS__);                                      \
            case 64: return FN<float, 64>(__VA_ARGS__);                                      \
            default: return FN<float, 128>(__VA_ARGS__);                                     \
        }                                                                                    \
    } while (0)

static int stream_setup(MuyoModel* m)
{
    if (!m->s_ok)
        return MUYO_OK;
    const Shape& s = m->s;
    std::vector<SLayer> sl(s.layers);
    for (int l = 0; l < s.layers; ++l) {
        const LayerPtrs w = layer_ptrs(m, l);
        sl[l] = SLayer{w.wqkv, w.bqkv, w.attn_norm, w.wo, w.ffn_norm, w.wgate, w.wup, w.wdown};
    }
    if (!m->d_slayers)
        MUYO_CUDA_TRY(cudaMalloc(&m->d_slayers, sizeof(SLayer) * s.layers));
    MUYO_CUDA_TRY(cudaMemcpy(m->d_slayers, sl.data(), sizeof(SLayer) * s.layers, cudaMemcpyHostToDevice));
    if (!m->ll) {
        const size_t words = (size_t)m->sa.ll_layer * s.layers + round16w(4 * (size_t)sm_count());
        MUYO_CUDA_TRY(cudaMalloc(&m->ll, words * sizeof(unsigned long long)));
        MUYO_CUDA_TRY(cudaMemset(m->ll, 0, words * sizeof(unsigned long long)));
    }
    MUYO_STREAM_DISPATCH(stream_setup_t, m);
}

template <typename KV, int HD>
static int launch_stream_t(MuyoModel* m, int prompt_end, int total, int n_steps, cudaStream_t st)
{
    SArgs a = m->sa;
    a.layers = m->d_slayers;
    a.embd = W(m, "token_embd.weight");
    a.lm = W(m, m->tied_output ? "token_embd.weight" : "output.weight");
    a.final_norm = F(m, "output_norm.weight");
    a.rope_cs = m->rope_cs;
    a.kc = m->kc;
    a.vc = m->vc;
    a.kv_layer_elems = (long long)(m->kv_layer_bytes / (m->s.kv_f16 ? 2 : 4));
    a.ll = m->ll;
    a.ll_best = m->ll + (size_t)a.ll_layer * m->s.layers;
    a.logits = m->logits;
    a.ctrl = m->ctrl;
    a.tokens = m->tokens;
    a.err = m->err;
    a.abort_g = m->abort_g;
    a.tag0 = m->s_tag;
    a.pos0 = m->host_pos;
    a.prompt_end = prompt_end;
    a.total = total;
    a.n_steps = n_steps;
    // Tags never repeat within 2^32 steps, and never take the value 0 the buffers start with.
    m->s_tag += (unsigned)n_steps;
    if (m->s_tag < (unsigned)n_steps)
        m->s_tag = 1;
    MUYO_CUDA_TRY(cudaMemsetAsync(m->abort_g, 0, sizeof(int), st));
    void* args[] = {&a};
    MUYO_CUDA_TRY(cudaLaunchCooperativeKernel((const void*)k_decode_stream<KV, HD>, dim3(m->s_grid), dim3(kSThreads),
                                              args, (size_t)m->s_smem, st));
    return MUYO_OK;
}

static int launch_stream(MuyoModel* m, int prompt_end, int total, int n_steps, cudaStream_t st)
{
    MUYO_STREAM_DISPATCH(launch_stream_t, m, prompt_end, total, n_steps, st);
}

__global__ void k_set_control(Control* c, Control v) { *c = v; }

}  // namespace muyo

using namespace muyo;

// ---- extern "C": KV append and op-level attention ----------------------------------------------------

template <typename KV, int HD>
__global__ void k_kv_append(int kv_heads, int max_seq, double base, const float* __restrict__ k,
                            const float* __restrict__ v, KV* __restrict__ kc, KV* __restrict__ vc,
                            const int32_t* __restrict__ pos_ptr)
{
    const int pos = *pos_ptr;
    if (pos < 0 || pos >= max_seq)
        return;  // a device position outside the cache: nothing is written
    const int h = blockIdx.x;
    const size_t row = ((size_t)h * max_seq + pos) * HD;
    for (int j = threadIdx.x; j < HD / 2; j += blockDim.x) {
        double c, s;
        rope_cs_f64(pos, j, HD, base, c, s);
        float y0, y1;
        rope_pair_f64(k[h * HD + j], k[h * HD + j + HD / 2], c, s, y0, y1);
        kc[row + j] = kv_round<KV>(y0);
        kc[row + j + HD / 2] = kv_round<KV>(y1);
    }
    for (int d = threadIdx.x; d < HD; d += blockDim.x)
        vc[row + d] = kv_round<KV>(v[h * HD + d]);
}

static int check_attn_params(const MuyoAttentionParams* p)
{
    MUYO_REQUIRE(p, "attention: null parameter block");
    MUYO_REQUIRE(p->heads > 0 && p->kv_heads > 0 && p->heads % p->kv_heads == 0,
                 "attention: heads %u must be a positive multiple of kv_heads %u", p->heads, p->kv_heads);
    MUYO_REQUIRE(p->heads / p->kv_heads <= (uint32_t)kAttnMaxGroup, "attention: more than %d query heads per KV head",
                 kAttnMaxGroup);
    if (!(p->head_dim == 16 || p->head_dim == 32 || p->head_dim == 64 || p->head_dim == 128)) {
        set_error("attention: head_dim %u not supported (16, 32, 64, 128)", p->head_dim);
        return MUYO_EUNSUPPORTED;
    }
    MUYO_REQUIRE(p->max_seq > 0, "attention: max_seq must be positive");
    MUYO_REQUIRE(p->kv_dtype == MUYO_KV_F32 || p->kv_dtype == MUYO_KV_F16, "attention: kv_dtype %u", p->kv_dtype);
    return MUYO_OK;
}

extern "C" size_t muyo_cuda_attention_workspace_size(const MuyoAttentionParams* p)
{
    if (!p || p->kv_heads == 0 || p->heads == 0)
        return 0;
    const size_t chunks = (p->max_seq + kAttnKeys - 1) / kAttnKeys;
    return (size_t)p->kv_heads * chunks * (p->heads / p->kv_heads) * (p->head_dim + 2) * sizeof(float);
}

template <typename KV, int HD>
static int launch_attention_op(const MuyoAttentionParams* q, const float* qv, const void* kc, const void* vc,
                               const int32_t* pos, float* out, float* part, cudaStream_t st)
{
    AttnDev p{(int)q->heads, (int)q->kv_heads, (int)(q->heads / q->kv_heads), (int)q->max_seq, (int)q->n_keys,
              q->scale, 0.0, (int)((q->max_seq + kAttnKeys - 1) / kAttnKeys), nullptr};
    const size_t smem = (size_t)attn_smem_floats(HD, p.gqa) * sizeof(float);
    auto k = k_attention<KV, HD, false, false>;
    if (smem > 48 * 1024)
        MUYO_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k<<<dim3(p.kv_heads, p.max_chunks), kAttnThreads, smem, st>>>(
        p, qv, const_cast<KV*>(static_cast<const KV*>(kc)), const_cast<KV*>(static_cast<const KV*>(vc)), pos, out, part,
        nullptr);
    MUYO_LAUNCH_CHECK();
    k_attention_combine<HD><<<p.kv_heads, kAttnThreads, 0, st>>>(p, pos, part, out);
    MUYO_LAUNCH_CHECK();
    return MUYO_OK;
}

extern "C" int muyo_cuda_attention_decode(const MuyoAttentionParams* p, const float* q, const void* k_cache,
                                          const void* v_cache, const int32_t* pos, float* out, void* workspace,
                                          size_t workspace_bytes, void* stream)
{
    clear_error();
    int rc = check_attn_params(p);
    if (rc)
        return rc;
    MUYO_REQUIRE(q && k_cache && v_cache && out, "attention: null buffer");
    MUYO_REQUIRE(pos || (p->n_keys > 0 && p->n_keys <= p->max_seq), "attention: n_keys %u must be in [1, max_seq %u]",
                 p->n_keys, p->max_seq);
    const size_t need = muyo_cuda_attention_workspace_size(p);
    MUYO_REQUIRE(workspace && workspace_bytes >= need, "attention: workspace of %zu bytes needed, %zu given", need,
                 workspace_bytes);
    const cudaStream_t st = as_stream(stream);
    float* part = static_cast<float*>(workspace);
    if (p->kv_dtype == MUYO_KV_F16) {
        switch (p->head_dim) {
            case 16: return launch_attention_op<__half, 16>(p, q, k_cache, v_cache, pos, out, part, st);
            case 32: return launch_attention_op<__half, 32>(p, q, k_cache, v_cache, pos, out, part, st);
            case 64: return launch_attention_op<__half, 64>(p, q, k_cache, v_cache, pos, out, part, st);
            default: return launch_attention_op<__half, 128>(p, q, k_cache, v_cache, pos, out, part, st);
        }
    }
    switch (p->head_dim) {
        case 16: return launch_attention_op<float, 16>(p, q, k_cache, v_cache, pos, out, part, st);
        case 32: return launch_attention_op<float, 32>(p, q, k_cache, v_cache, pos, out, part, st);
        case 64: return launch_attention_op<float, 64>(p, q, k_cache, v_cache, pos, out, part, st);
        default: return launch_attention_op<float, 128>(p, q, k_cache, v_cache, pos, out, part, st);
    }
}

extern "C" int muyo_cuda_kv_append(const MuyoAttentionParams* p, float rope_base, const float* k, const float* v,
                                   void* k_cache, void* v_cache, const int32_t* pos, void* stream)
{
    clear_error();
    int rc = check_attn_params(p);
    if (rc)
        return rc;
    MUYO_REQUIRE(k && v && k_cache && v_cache && pos, "kv_append: null buffer");
    MUYO_REQUIRE(rope_base > 0.0f, "kv_append: rope_base must be positive");
    const cudaStream_t st = as_stream(stream);
    const int kvh = (int)p->kv_heads, S = (int)p->max_seq;
#define MUYO_KV_APPEND(KV, HD)                                                                            \
    k_kv_append<KV, HD><<<kvh, 64, 0, st>>>(kvh, S, (double)rope_base, k, v, static_cast<KV*>(k_cache), \
                                            static_cast<KV*>(v_cache), pos)
    if (p->kv_dtype == MUYO_KV_F16) {
        if (p->head_dim == 16) MUYO_KV_APPEND(__half, 16);
        else if (p->head_dim == 32) MUYO_KV_APPEND(__half, 32);
        else if (p->head_dim == 64) MUYO_KV_APPEND(__half, 64);
        else MUYO_KV_APPEND(__half, 128);
    } else {
        if (p->head_dim == 16) MUYO_KV_APPEND(float, 16);
        else if (p->head_dim == 32) MUYO_KV_APPEND(float, 32);
        else if (p->head_dim == 64) MUYO_KV_APPEND(float, 64);
        else MUYO_KV_APPEND(float, 128);
    }
#undef MUYO_KV_APPEND
    MUYO_LAUNCH_CHECK();
    return MUYO_OK;
}

// ---- extern "C": one layer -----------------------------------------------------------------------------

extern "C" size_t muyo_cuda_layer_workspace_size(const MuyoQwen2Config* c)
{
    Shape s{};
    if (make_shape(c, s, false) != MUYO_OK)
        return 0;
    return layer_scratch_bytes(s);
}

extern "C" int muyo_cuda_layer_step(const MuyoQwen2Config* c, const MuyoLayerWeights* w, void* k_cache, void* v_cache,
                                    const int32_t* pos, const float* x_in, float* x_out, void* workspace,
                                    size_t workspace_bytes, void* stream)
{
    clear_error();
    Shape s{};
    int rc = make_shape(c, s, false);
    if (rc)
        return rc;
    MUYO_REQUIRE(w && w->attn_norm && w->wqkv && w->bqkv && w->wo && w->ffn_norm && w->wgate && w->wup && w->wdown,
                 "layer_step: null weight pointer");
    MUYO_REQUIRE(k_cache && v_cache && pos && x_in && x_out, "layer_step: null buffer");
    MUYO_REQUIRE(x_in != x_out, "layer_step: x_in and x_out must not alias");
    MUYO_REQUIRE(aligned16(w->wqkv) && aligned16(w->wo) && aligned16(w->wgate) && aligned16(w->wup) &&
                     aligned16(w->wdown),
                 "layer_step: weight matrices must be 16-byte aligned");
    MUYO_REQUIRE(aligned16(w->attn_norm) && aligned16(w->ffn_norm) && aligned16(x_in) && aligned16(x_out),
                 "layer_step: norm weights, x_in and x_out must be 16-byte aligned");
    const size_t need = layer_scratch_bytes(s);
    MUYO_REQUIRE(workspace && workspace_bytes >= need, "layer_step: workspace of %zu bytes needed, %zu given", need,
                 workspace_bytes);
    MUYO_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255u) == 0, "layer_step: workspace must be 256-byte aligned");
    LayerPtrs lp{w->attn_norm,
                 static_cast<const __half*>(w->wqkv),
                 w->bqkv,
                 static_cast<const __half*>(w->wo),
                 w->ffn_norm,
                 static_cast<const __half*>(w->wgate),
                 static_cast<const __half*>(w->wup),
                 static_cast<const __half*>(w->wdown)};
    return layer_forward(s, lp, k_cache, v_cache, pos, x_in, x_out, carve_layer_scratch(s, workspace), nullptr, nullptr,
                         nullptr, nullptr, as_stream(stream), false);
}

// ---- extern "C": model ---------------------------------------------------------------------------------

static void free_model(MuyoModel* m)
{
    if (!m)
        return;
    if (m->exec)
        cudaGraphExecDestroy(m->exec);
    if (m->graph)
        cudaGraphDestroy(m->graph);
    if (m->exec_n)
        cudaGraphExecDestroy(m->exec_n);
    if (m->graph_n)
        cudaGraphDestroy(m->graph_n);
    if (m->cap_stream)
        cudaStreamDestroy(m->cap_stream);
    cudaFree(m->rope_cs);
    cudaFree(m->d_slayers);
    cudaFree(m->ll);
    cudaFree(m->arena);
    cudaFree(m->kc);
    cudaFree(m->vc);
    cudaFree(m->scratch);
    cudaFree(m->rng);
    cudaFree(m->pf_buf);
    if (m->pinned)
        cudaFreeHost(m->pinned);
    delete m;
}

extern "C" int muyo_model_create(const MuyoQwen2Config* c, int device, MuyoModel** out)
{
    clear_error();
    MUYO_REQUIRE(out, "model_create: out is null");
    *out = nullptr;
    Shape s{};
    int rc = make_shape(c, s, true);
    if (rc)
        return rc;
    MUYO_REQUIRE(s.layers > 0, "model_create: layers must be positive");
    MUYO_CUDA_TRY(cudaSetDevice(device));
    MuyoModel* m = new (std::nothrow) MuyoModel();
    if (!m) {
        set_error("model_create: host allocation failed");
        return MUYO_ENOMEM;
    }
    m->s = s;
    m->device = device;
    // Weight arena layout (256-byte aligned slots). QKV weights and biases are stacked by rows so one
    // GEMV produces q, k and v; the GGUF tensors attn_{q,k,v}.{weight,bias} land in row ranges of it.
    size_t off = 0;
    auto slot = [&](const std::string& name, size_t elems, bool f16) {
        m->slots[name] = TensorSlot{off, elems * (f16 ? 2 : 4), f16, false};
        off += align256(elems * (f16 ? 2 : 4));
    };
    const size_t H = s.hidden, Fd = s.ffn, V = s.vocab;
    slot("token_embd.weight", V * H, true);
    slot("output.weight", 0, true);  // tied unless set
    slot("output_norm.weight", H, false);
    for (int l = 0; l < s.layers; ++l) {
        const std::string p = "blk." + std::to_string(l) + ".";
        slot(p + "attn_norm.weight", H, false);
        slot(p + "attn_qkv.weight", (size_t)s.qkv_rows * H, true);
        slot(p + "attn_qkv.bias", s.qkv_rows, false);
        slot(p + "attn_output.weight", H * s.q_dim, true);
        slot(p + "ffn_norm.weight", H, false);
        slot(p + "ffn_gate.weight", Fd * H, true);
        slot(p + "ffn_up.weight", Fd * H, true);
        slot(p + "ffn_down.weight", H * Fd, true);
    }
    m->arena_bytes = off;
    cudaError_t e = cudaMalloc(&m->arena, off);
    m->kv_layer_bytes = align256((size_t)s.kv_heads * s.max_seq * s.head_dim * (s.kv_f16 ? 2 : 4));
    if (e == cudaSuccess)
        e = cudaMalloc(&m->kc, m->kv_layer_bytes * s.layers);
    if (e == cudaSuccess)
        e = cudaMalloc(&m->vc, m->kv_layer_bytes * s.layers);
    m->lm_grid = sm_count() * 8;
    const size_t scratch_bytes = layer_scratch_bytes(s) + align256(sizeof(float) * H) + align256(sizeof(float) * V) +
                                 align256(sizeof(Pair) * m->lm_grid) + align256(sizeof(int32_t)) +
                                 align256(sizeof(Control)) + align256(sizeof(int32_t) * s.max_seq) +
                                 align256(sizeof(unsigned)) + align256(sizeof(int));
    if (e == cudaSuccess)
        e = cudaMalloc(&m->scratch, scratch_bytes);
    if (e == cudaSuccess)
        e = cudaMemset(m->scratch, 0, scratch_bytes);
    if (e == cudaSuccess)
        e = cudaMemset(m->kc, 0, m->kv_layer_bytes * s.layers);
    if (e == cudaSuccess)
        e = cudaMemset(m->vc, 0, m->kv_layer_bytes * s.layers);
    m->pinned_ints = (size_t)s.max_seq + 16;
    if (e == cudaSuccess)
        e = cudaMallocHost(&m->pinned, m->pinned_ints * sizeof(int32_t));
    if (e == cudaSuccess)
        e = cudaStreamCreateWithFlags(&m->cap_stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        set_error("model_create: %s", cudaGetErrorString(e));
        free_model(m);
        return e == cudaErrorMemoryAllocation ? MUYO_ENOMEM : MUYO_ECUDA;
    }
    char* p = m->scratch;
    m->ls = carve_layer_scratch(s, p);
    p += layer_scratch_bytes(s);
    m->h = reinterpret_cast<float*>(p);
    p += align256(sizeof(float) * H);
    m->logits = reinterpret_cast<float*>(p);
    p += align256(sizeof(float) * V);
    m->lm_part = reinterpret_cast<Pair*>(p);
    p += align256(sizeof(Pair) * m->lm_grid);
    m->lm_counter = reinterpret_cast<int32_t*>(p);
    p += align256(sizeof(int32_t));
    m->ctrl = reinterpret_cast<Control*>(p);
    p += align256(sizeof(Control));
    m->tokens = reinterpret_cast<int32_t*>(p);
    p += align256(sizeof(int32_t) * s.max_seq);
    m->abort_g = reinterpret_cast<int*>(p);
    p += align256(sizeof(int));
    m->err = reinterpret_cast<int*>(p);
    *out = m;
    return MUYO_OK;
}

static bool split_qkv(const std::string& name, std::string& base, int& part, bool& bias)
{
    // blk.N.attn_{q,k,v}.{weight,bias} -> blk.N.attn_qkv.{weight,bias}, part 0/1/2
    const size_t a = name.find(".attn_");
    if (a == std::string::npos || name.size() < a + 8)
        return false;
    const char which = name[a + 6];
    if (name[a + 7] != '.' || (which != 'q' && which != 'k' && which != 'v'))
        return false;
    const std::string rest = name.substr(a + 8);
    if (rest != "weight" && rest != "bias")
        return false;
    bias = rest == "bias";
    base = name.substr(0, a) + ".attn_qkv." + rest;
    part = which == 'q' ? 0 : which == 'k' ? 1 : 2;
    return true;
}

extern "C" int muyo_model_set_tensor(MuyoModel* m, const char* name, const void* host, size_t bytes)
{
    clear_error();
    MUYO_REQUIRE(m && name && host, "set_tensor: null argument");
    MUYO_CUDA_TRY(cudaSetDevice(m->device));
    const Shape& s = m->s;
    std::string n(name), base;
    int part = 0;
    bool bias = false;
    if (split_qkv(n, base, part, bias)) {
        auto it = m->slots.find(base);
        MUYO_REQUIRE(it != m->slots.end(), "set_tensor: unknown tensor %s", name);
        const size_t per_row = bias ? 4 : (size_t)s.hidden * 2;
        const size_t row0 = part == 0 ? 0 : part == 1 ? s.q_dim : (size_t)s.q_dim + s.kv_dim;
        const size_t rows = part == 0 ? s.q_dim : s.kv_dim;
        MUYO_REQUIRE(bytes == rows * per_row, "set_tensor: %s has %zu bytes, expected %zu", name, bytes, rows * per_row);
        MUYO_CUDA_TRY(cudaMemcpy(m->arena + it->second.offset + row0 * per_row, host, bytes, cudaMemcpyHostToDevice));
        // A stacked slot counts as set once all three parts arrived.
        m->slots[base + "#" + std::to_string(part)] = TensorSlot{0, 0, false, true};
        return MUYO_OK;
    }
    if (n == "output.weight") {
        const size_t need = (size_t)s.vocab * s.hidden * 2;
        MUYO_REQUIRE(bytes == need, "set_tensor: output.weight has %zu bytes, expected %zu", bytes, need);
        // Untie: give the LM head its own copy at the end of a fresh arena slot.
        char* extra = nullptr;
        MUYO_CUDA_TRY(cudaMalloc(&extra, m->arena_bytes + align256(need)));
        MUYO_CUDA_TRY(cudaMemcpy(extra, m->arena, m->arena_bytes, cudaMemcpyDeviceToDevice));
        cudaFree(m->arena);
        m->arena = extra;
        m->slots["output.weight"] = TensorSlot{m->arena_bytes, need, true, true};
        m->arena_bytes += align256(need);
        MUYO_CUDA_TRY(cudaMemcpy(m->arena + m->slots["output.weight"].offset, host, bytes, cudaMemcpyHostToDevice));
        m->tied_output = false;
        m->finalized = false;
        return MUYO_OK;
    }
    auto it = m->slots.find(n);
    MUYO_REQUIRE(it != m->slots.end() && n.find("attn_qkv") == std::string::npos, "set_tensor: unknown tensor %s",
                 name);
    MUYO_REQUIRE(bytes == it->second.bytes, "set_tensor: %s has %zu bytes, expected %zu", name, bytes,
                 it->second.bytes);
    MUYO_CUDA_TRY(cudaMemcpy(m->arena + it->second.offset, host, bytes, cudaMemcpyHostToDevice));
    it->second.set = true;
    return MUYO_OK;
}

// (Re)records the decode-step graph.
constexpr int kGraphSteps = 8;

// Captures `steps` decode steps into one graph (a step is position-invariant: the position and the
// fed token live in device memory).
static int capture_steps(MuyoModel* m, int steps, cudaGraph_t& graph, cudaGraphExec_t& exec)
{
    if (exec) {
        cudaGraphExecDestroy(exec);
        exec = nullptr;
    }
    if (graph) {
        cudaGraphDestroy(graph);
        graph = nullptr;
    }
    MUYO_CUDA_TRY(cudaStreamBeginCapture(m->cap_stream, cudaStreamCaptureModeThreadLocal));
    int rc = MUYO_OK;
    for (int i = 0; i < steps && rc == MUYO_OK; ++i)
        rc = record_step(m, m->cap_stream);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(m->cap_stream, &g);
    if (rc != MUYO_OK) {
        if (g)
            cudaGraphDestroy(g);
        return rc;
    }
    MUYO_CUDA_TRY(e);
    graph = g;
    MUYO_CUDA_TRY(cudaGraphInstantiate(&exec, g, 0));
    return MUYO_OK;
}

static int record_graph(MuyoModel* m)
{
    const int rc = capture_steps(m, 1, m->graph, m->exec);
    return rc != MUYO_OK ? rc : capture_steps(m, kGraphSteps, m->graph_n, m->exec_n);
}

extern "C" int muyo_model_finalize(MuyoModel* m, void* stream)
{
    clear_error();
    MUYO_REQUIRE(m, "finalize: null model");
    MUYO_CUDA_TRY(cudaSetDevice(m->device));
    for (const auto& kv : m->slots) {
        const std::string& n = kv.first;
        if (n.find('#') != std::string::npos || n == "output.weight")
            continue;
        if (n.find("attn_qkv") != std::string::npos) {
            for (int part = 0; part < 3; ++part)
                MUYO_REQUIRE(m->slots.count(n + "#" + std::to_string(part)), "finalize: %s part %d was never set",
                             n.c_str(), part);
            continue;
        }
        MUYO_REQUIRE(kv.second.set, "finalize: tensor %s was never set", n.c_str());
    }
    (void)stream;
    const Shape& s = m->s;
    // (cos, sin) of theta = pos * base^(-2j/hd) in float64 (tools/reference_qwen2.py:88-89), per position.
    if (!m->rope_cs) {
        std::vector<double> cs((size_t)s.max_seq * s.head_dim);
        for (int pos = 0; pos < s.max_seq; ++pos)
            for (int j = 0; j < s.head_dim / 2; ++j) {
                const double theta = (double)pos * std::pow((double)s.rope_base, -2.0 * j / s.head_dim);
                cs[(size_t)pos * s.head_dim + j] = std::cos(theta);
                cs[(size_t)pos * s.head_dim + s.head_dim / 2 + j] = std::sin(theta);
            }
        MUYO_CUDA_TRY(cudaMalloc(&m->rope_cs, cs.size() * sizeof(double)));
        MUYO_CUDA_TRY(cudaMemcpy(m->rope_cs, cs.data(), cs.size() * sizeof(double), cudaMemcpyHostToDevice));
        m->s.rope_cs = m->rope_cs;
    }
    {
        int rc = stream_plan(m);
        if (rc == MUYO_OK)
            rc = stream_setup(m);
        if (rc)
            return rc;
    }
    const int rc = record_graph(m);
    if (rc)
        return rc;
    m->finalized = true;
    return MUYO_OK;
}

extern "C" int muyo_model_reset(MuyoModel* m, void* stream)
{
    clear_error();
    MUYO_REQUIRE(m, "reset: null model");
    MUYO_CUDA_TRY(cudaSetDevice(m->device));
    const cudaStream_t st = as_stream(stream);
    MUYO_CUDA_TRY(cudaMemsetAsync(m->kc, 0, m->kv_layer_bytes * m->s.layers, st));
    MUYO_CUDA_TRY(cudaMemsetAsync(m->vc, 0, m->kv_layer_bytes * m->s.layers, st));
    MUYO_CUDA_TRY(cudaMemsetAsync(m->ctrl, 0, sizeof(Control), st));
    MUYO_CUDA_TRY(cudaStreamSynchronize(st));
    m->host_pos = 0;
    return MUYO_OK;
}

// Sets the control block for `n_steps` steps starting at the current position, with prompt ids
// forced up to `prompt_end`, and runs n_steps steps: the kGraphSteps-step graph while that many are
// left, then the one-step graph.
static int run_steps(MuyoModel* m, int prompt_end, int total, int n_steps, cudaStream_t st)
{
    if (m->engine == 0 && m->sampling) {
        set_error("decode: the device sampler runs in the graph engine (engine 1), not the persistent kernel");
        return MUYO_EUNSUPPORTED;
    }
    if (m->engine == 0 && !m->s_ok) {
        set_error("decode: the persistent kernel does not take these shapes (%s); use the graph engine (engine 1)",
                  m->s_why.c_str());
        return MUYO_EUNSUPPORTED;
    }
    const bool persistent = m->engine == 0;
    k_set_control<<<1, 1, 0, st>>>(m->ctrl, Control{m->host_pos, prompt_end, total, 0});
    MUYO_LAUNCH_CHECK();
    if (persistent) {
        const int rc = launch_stream(m, prompt_end, total, n_steps, st);
        if (rc)
            return rc;
    } else {
        int i = 0;
        for (; i + kGraphSteps <= n_steps; i += kGraphSteps)
            MUYO_CUDA_TRY(cudaGraphLaunch(m->exec_n, st));
        for (; i < n_steps; ++i)
            MUYO_CUDA_TRY(cudaGraphLaunch(m->exec, st));
    }
    m->host_pos += n_steps;
    return MUYO_OK;
}

// Error word of the decode kernels (read after a synchronisation); clears it.
static int check_device_error(MuyoModel* m, cudaStream_t st)
{
    int e = 0;
    MUYO_CUDA_TRY(cudaMemcpyAsync(&e, m->err, sizeof(int), cudaMemcpyDeviceToHost, st));
    MUYO_CUDA_TRY(cudaStreamSynchronize(st));
    if (e != 0) {
        MUYO_CUDA_TRY(cudaMemsetAsync(m->err, 0, sizeof(int), st));
        set_error("decode: a bounded device wait expired (error word %d: 3 persistent kernel, 4 weight-tile copy, "
                  "6 prefill tensor-core pipeline)",
                  e);
        return MUYO_ETIMEOUT;
    }
    return MUYO_OK;
}

// ---- batched prefill ---------------------------------------------------------------------------------

constexpr int kPfCapMax = 1024;  // largest "prefill_positions" (longer prompts take several passes)
constexpr int kPfMaxSplits = 16;

// TMA descriptors of one tcgen05 prefill GEMM: the W rows (two matrices for gate | up) and the
// activation halves.
struct PfMaps {
    CUtensorMap w0, w1, xhi, xlo;
};

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against the driver).
static EncodeTiledFn encode_tiled()
{
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
        else
            cudaGetLastError();
    });
    return fn;
}

// F16 matrix [rows][cols] with row stride ld halves, read in boxes of 64 halves x box_rows rows with
// the 128-byte swizzle (the tcgen05 GEMM's operand layout; outside the matrix the box is zero-filled).
// cols, ld multiples of 8; base 16-byte aligned.
static int make_map(CUtensorMap* map, const void* base, int cols, int rows, int ld, int box_rows)
{
    EncodeTiledFn fn = encode_tiled();
    if (!fn) {
        set_error("prefill: cuTensorMapEncodeTiled is not available from the driver");
        return MUYO_EUNSUPPORTED;
    }
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kTcBK, (cuuint32_t)box_rows};  // 128-byte rows, swizzled
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("prefill: cuTensorMapEncodeTiled failed (%d) for a %d x %d matrix", (int)r, rows, cols);
        return MUYO_ECUDA;
    }
    return MUYO_OK;
}

static int pf_alloc(MuyoModel* m)
{
    if (m->pf_buf)
        return MUYO_OK;
    const Shape& s = m->s;
    const size_t wide = (size_t)std::max(std::max(s.hidden, s.q_dim), s.ffn);
    const size_t part = (size_t)kPfMaxSplits * (size_t)m->pf_cap * std::max(s.qkv_rows, s.hidden);
    const size_t f32 = (size_t)m->pf_cap * ((size_t)s.hidden + s.qkv_rows + 2 * (size_t)s.q_dim + 2 * (size_t)s.ffn) + part;
    const size_t bytes = f32 * sizeof(float) + 2 * (size_t)m->pf_cap * wide * sizeof(__half) + 256 * 9;
    if (cudaMalloc(&m->pf_buf, bytes) != cudaSuccess) {
        cudaGetLastError();
        m->pf_buf = nullptr;
        set_error("prefill: cannot allocate %zu bytes of activations", bytes);
        return MUYO_ENOMEM;
    }
    char* p = m->pf_buf;
    auto take = [&](size_t n) {
        char* r = p;
        p += (n + 255) / 256 * 256;
        return r;
    };
    m->pf_x = reinterpret_cast<float*>(take((size_t)m->pf_cap * s.hidden * 4));
    m->pf_qkv = reinterpret_cast<float*>(take((size_t)m->pf_cap * s.qkv_rows * 4));
    m->pf_q = reinterpret_cast<float*>(take((size_t)m->pf_cap * s.q_dim * 4));
    m->pf_att = reinterpret_cast<float*>(take((size_t)m->pf_cap * s.q_dim * 4));
    m->pf_gu = reinterpret_cast<float*>(take((size_t)m->pf_cap * 2 * s.ffn * 4));
    m->pf_hi = reinterpret_cast<__half*>(take((size_t)m->pf_cap * wide * 2));
    m->pf_lo = reinterpret_cast<__half*>(take((size_t)m->pf_cap * wide * 2));
    m->pf_part = reinterpret_cast<float*>(take(part * 4));
    m->pf_part_floats = part;
    if ((size_t)(p - m->pf_buf) > bytes + 256 * 9) {
        set_error("prefill: buffer plan overflow");
        return MUYO_EINVAL;
    }
    for (auto k : {k_pf_gemm<PF_STORE>, k_pf_gemm<PF_BIAS>, k_pf_gemm<PF_ADD>})
        MUYO_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPfGemmSmem));
    for (auto k : {k_pf_gemm_tc<PF_STORE>, k_pf_gemm_tc<PF_BIAS>, k_pf_gemm_tc<PF_ADD>})
        MUYO_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem));
    return MUYO_OK;
}

// K-range splits of a prefill GEMM: enough CTAs for two per SM, each range at least 4 stages long.
// tc: the tensor-core kernel's 128-row tiles (else the warp-MMA kernel's 64-row tiles).
// (tc: the persistent kernel's work items, enough for every SM.)
static int pf_splits(int N, int K, int T, bool tc = false)
{
    const int bm = tc ? kTcBM : kPfBM, bn = tc ? kTcBN : kPfBN;
    const int ctas = ((N + bm - 1) / bm) * ((T + bn - 1) / bn);
    const int stages = (K + kPfBK - 1) / kPfBK;
    // mma.sync: enough CTAs for two per SM. tcgen05 (persistent, one CTA per SM): the most splits
    // that still fit one wave, so long passes do not pay a second partial wave and a larger
    // reduction (fewer K stages per item than 2 would not amortise the pipeline ramp).
    int S = tc ? std::max(1, sm_count() / ctas) : (2 * sm_count() + ctas - 1) / ctas;
    S = std::min(S, std::max(1, stages / (tc ? 2 : 4)));
    return std::max(1, std::min(S, kPfMaxSplits));
}

// part: S * T * N floats when pf_splits > 1 (the prefill workspace). tc: the tensor maps of the
// tcgen05 kernel (its W rows: n_split a multiple of 128), else the warp-level mma.sync kernel runs.
// err: the bounded waits' error word (may be null).
template <int EPI>
static int pf_gemm(const __half* w0, const __half* w1, int n_split, int N, int K, int T, const __half* xhi,
                   const __half* xlo, int ldx, float* y, int ldy, const float* bias, float* part, size_t part_floats,
                   cudaStream_t st, const PfMaps* tc = nullptr, int* err = nullptr)
{
    PfGemm g{w0, w1 ? w1 : w0, n_split, N, K, T, xhi, xlo, ldx, y, ldy, bias};
    int S = pf_splits(N, K, T, tc != nullptr);
    if ((size_t)S * T * N > part_floats)
        S = 1;
    if (tc) {  // persistent: one CTA per SM at most, striding over (feature tile, position tile, K range)
        const int items = ((N + kTcBM - 1) / kTcBM) * ((T + kTcBN - 1) / kTcBN) * S;
        MUYO_CUDA_TRY(launch_kernel(k_pf_gemm_tc<EPI>, dim3(std::min(items, sm_count())), dim3(kTcThreads), kTcSmem, st,
                                    true, g, part, err, S, tc->w0, tc->w1, tc->xhi, tc->xlo));
    } else {
        const dim3 grid((N + kPfBM - 1) / kPfBM, (T + kPfBN - 1) / kPfBN, S);
        MUYO_CUDA_TRY(launch_kernel(k_pf_gemm<EPI>, grid, dim3(kPfThreads), kPfGemmSmem, st, true, g, part));
    }
    if (S > 1) {
        const int blocks = (int)std::min<size_t>(((size_t)T * N + 255) / 256, (size_t)sm_count() * 8);
        MUYO_CUDA_TRY(launch_kernel(k_pf_reduce<EPI>, dim3(blocks), dim3(256), 0, st, true, g, (const float*)part, S));
    }
    return MUYO_OK;
}

template <typename KV, int HD>
static int pf_attention_t(const Shape& s, float* q, float* out, const float* qkv, char* kc, char* vc, int p0, int T,
                          cudaStream_t st)
{
    PfRope r{qkv, s.qkv_rows, q, p0, s.heads, s.kv_heads, s.max_seq, s.rope_cs};
    MUYO_CUDA_TRY(launch_kernel(k_pf_rope_append<KV, HD>, dim3(T, s.heads + s.kv_heads), dim3(HD), 0, st, true, r,
                                reinterpret_cast<KV*>(kc), reinterpret_cast<KV*>(vc)));
    PfAttn a{q, out, p0, s.heads, s.kv_heads, s.gqa, s.max_seq, 1.0f / sqrtf((float)s.head_dim)};
    if constexpr (std::is_same<KV, __half>::value && (HD == 64 || HD == 128)) {
        // F16 cache: the tensor-core kernel, one CTA per (64-position query tile, query head).
        constexpr size_t fsmem = pf_flash_smem<HD>();
        if (fsmem > 48 * 1024)
            MUYO_CUDA_TRY(cudaFuncSetAttribute(k_pf_flash<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fsmem));
        MUYO_CUDA_TRY(launch_kernel(k_pf_flash<HD>, dim3((T + kPfFlashRows - 1) / kPfFlashRows, s.heads),
                                    dim3(kPfFlashThreads), fsmem, st, true, a, T, reinterpret_cast<const __half*>(kc),
                                    reinterpret_cast<const __half*>(vc)));
        return MUYO_OK;
    }
    const size_t smem = pf_attn_smem(HD, s.gqa);
    if (smem > 48 * 1024)
        MUYO_CUDA_TRY(cudaFuncSetAttribute(k_pf_attention<KV, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    MUYO_CUDA_TRY(launch_kernel(k_pf_attention<KV, HD>, dim3(s.kv_heads, T), dim3(kPfAttnThreads), smem, st, true, a,
                                reinterpret_cast<const KV*>(kc), reinterpret_cast<const KV*>(vc)));
    return MUYO_OK;
}

static int pf_attention(const Shape& s, float* q, float* out, const float* qkv, char* kc, char* vc, int p0, int T,
                        cudaStream_t st)
{
#define MUYO_PF_ATTN(KV)                                                                        switch (s.head_dim) {                                                                           case 16: return pf_attention_t<KV, 16>(s, q, out, qkv, kc, vc, p0, T, st);                  case 32: return pf_attention_t<KV, 32>(s, q, out, qkv, kc, vc, p0, T, st);                  case 64: return pf_attention_t<KV, 64>(s, q, out, qkv, kc, vc, p0, T, st);                  default: return pf_attention_t<KV, 128>(s, q, out, qkv, kc, vc, p0, T, st);             }
    if (s.kv_f16)
        MUYO_PF_ATTN(__half)
    MUYO_PF_ATTN(float)
#undef MUYO_PF_ATTN
}

// The tcgen05 prefill's tensor maps: per layer qkv, o, gate, up, down (W row tiles of 128), then the
// activation halves as K = hidden, q_dim and ffn wide (position tiles of 64).
static int pf_make_maps(MuyoModel* m)
{
    const Shape& s = m->s;
    const int H = s.hidden, QD = s.q_dim, F = s.ffn, ldh = std::max(std::max(H, QD), F);
    std::vector<CUtensorMap> maps((size_t)5 * s.layers + 6);
    int rc;
    for (int l = 0; l < s.layers; ++l) {
        const LayerPtrs w = layer_ptrs(m, l);
        CUtensorMap* lm = maps.data() + (size_t)5 * l;
        if ((rc = make_map(&lm[0], w.wqkv, H, s.qkv_rows, H, kTcBM)) || (rc = make_map(&lm[1], w.wo, QD, H, QD, kTcBM)) ||
            (rc = make_map(&lm[2], w.wgate, H, F, H, kTcBM)) || (rc = make_map(&lm[3], w.wup, H, F, H, kTcBM)) ||
            (rc = make_map(&lm[4], w.wdown, F, H, F, kTcBM)))
            return rc;
    }
    CUtensorMap* xm = maps.data() + (size_t)5 * s.layers;
    const int ks[3] = {H, QD, F};
    for (int i = 0; i < 3; ++i)
        if ((rc = make_map(&xm[2 * i], m->pf_hi, ks[i], m->pf_cap, ldh, kTcBN)) ||
            (rc = make_map(&xm[2 * i + 1], m->pf_lo, ks[i], m->pf_cap, ldh, kTcBN)))
            return rc;
    m->pf_maps.swap(maps);
    return MUYO_OK;
}

// Positions [p0, p0 + n) of m->tokens through every layer: their keys and values go to the cache.
// No logits are formed (the decode step at position p0 + n forms the next ones).
static int prefill_run(MuyoModel* m, int p0, int n, cudaStream_t st)
{
    const Shape& s = m->s;
    const int H = s.hidden, QD = s.q_dim, F = s.ffn;
    const int ldh = std::max(std::max(H, QD), F);
    int rc;
    if (m->pf_tc && m->pf_maps.empty() && (rc = pf_make_maps(m)))
        return rc;
    // tcgen05 GEMM of layer l: weight maps a and b of the layer (b for rows past the split) and the
    // activation halves of K index xk (hidden, q_dim, ffn); null selects the mma.sync kernel. Per
    // GEMM (pf_tc 2): tcgen05 from 256 positions, or for matrices of 4M weights and more, where it
    // measured faster; below that the mma.sync kernel's shorter set-up wins.
    PfMaps pm;
    auto tc = [&](int l, int a, int b, int xk, int N, int K, int T) -> const PfMaps* {
        const bool use = m->pf_tc == 1 || (m->pf_tc == 2 && (T >= 256 || (size_t)N * K >= ((size_t)4 << 20)));
        if (!use || (a != b && F % kTcBM != 0))
            return nullptr;
        const CUtensorMap* lm = m->pf_maps.data() + (size_t)5 * l;
        const CUtensorMap* xm = m->pf_maps.data() + (size_t)5 * s.layers + 2 * xk;
        pm = PfMaps{lm[a], lm[b], xm[0], xm[1]};
        return &pm;
    };
    for (int c0 = 0; c0 < n; c0 += m->pf_cap) {
        const int T = std::min(m->pf_cap, n - c0), pos0 = p0 + c0;
        MUYO_CUDA_TRY(launch_kernel(k_pf_embed, dim3(T), dim3(256), 0, st, true, W(m, "token_embd.weight"),
                                    (const int32_t*)(m->tokens + pos0), s.vocab, H, m->pf_x));
        for (int l = 0; l < s.layers; ++l) {
            const LayerPtrs w = layer_ptrs(m, l);
            char* kc = static_cast<char*>(m->kc) + m->kv_layer_bytes * l;
            char* vc = static_cast<char*>(m->vc) + m->kv_layer_bytes * l;
            MUYO_CUDA_TRY(launch_kernel(k_pf_norm_split, dim3(T), dim3(256), 0, st, true, (const float*)m->pf_x, H,
                                        w.attn_norm, s.eps, H, m->pf_hi, m->pf_lo, ldh));
            if ((rc = pf_gemm<PF_BIAS>(w.wqkv, nullptr, s.qkv_rows, s.qkv_rows, H, T, m->pf_hi, m->pf_lo, ldh,
                                       m->pf_qkv, s.qkv_rows, w.bqkv, m->pf_part, m->pf_part_floats, st, tc(l, 0, 0, 0, s.qkv_rows, H, T),
                                       m->err)))
                return rc;
            if ((rc = pf_attention(s, m->pf_q, m->pf_att, m->pf_qkv, kc, vc, pos0, T, st)))
                return rc;
            MUYO_CUDA_TRY(launch_kernel(k_pf_split, dim3(T), dim3(256), 0, st, true, (const float*)m->pf_att, QD, QD,
                                        m->pf_hi, m->pf_lo, ldh));
            if ((rc = pf_gemm<PF_ADD>(w.wo, nullptr, H, H, QD, T, m->pf_hi, m->pf_lo, ldh, m->pf_x, H, nullptr, m->pf_part,
                                      m->pf_part_floats, st, tc(l, 1, 1, 1, H, QD, T), m->err)))
                return rc;
            MUYO_CUDA_TRY(launch_kernel(k_pf_norm_split, dim3(T), dim3(256), 0, st, true, (const float*)m->pf_x, H,
                                        w.ffn_norm, s.eps, H, m->pf_hi, m->pf_lo, ldh));
            if ((rc = pf_gemm<PF_STORE>(w.wgate, w.wup, F, 2 * F, H, T, m->pf_hi, m->pf_lo, ldh, m->pf_gu, 2 * F,
                                        nullptr, m->pf_part, m->pf_part_floats, st, tc(l, 2, 3, 0, 2 * F, H, T), m->err)))
                return rc;
            MUYO_CUDA_TRY(launch_kernel(k_pf_swiglu_split, dim3(T), dim3(256), 0, st, true, (const float*)m->pf_gu, F,
                                        m->pf_hi, m->pf_lo, ldh));
            if ((rc = pf_gemm<PF_ADD>(w.wdown, nullptr, H, H, F, T, m->pf_hi, m->pf_lo, ldh, m->pf_x, H, nullptr, m->pf_part,
                                      m->pf_part_floats, st, tc(l, 4, 4, 2, H, F, T), m->err)))
                return rc;
        }
    }
    MUYO_LAUNCH_CHECK();
    return MUYO_OK;
}

// generate: with batched prefill, every prompt position but the last goes through prefill_run;
// returns the number of positions it fed (0 when prefill is off or the prompt has one id).
static int feed_prompt(MuyoModel* m, int n_prompt, cudaStream_t st, int& fed)
{
    fed = 0;
    if (!m->prefill || n_prompt < 2)
        return MUYO_OK;
    const int rc = prefill_run(m, m->host_pos, n_prompt - 1, st);
    if (rc)
        return rc;
    fed = n_prompt - 1;
    m->host_pos += fed;
    return MUYO_OK;
}

static int check_generate(MuyoModel* m, int n_prompt, int n_predict)
{
    MUYO_REQUIRE(m, "generate: null model");
    if (!m->finalized) {
        set_error("generate: model not finalized");
        return MUYO_ESTATE;
    }
    MUYO_REQUIRE(n_prompt >= 1 && n_predict >= 0, "generate: need n_prompt >= 1 and n_predict >= 0");
    if ((long long)m->host_pos + n_prompt + n_predict > m->s.max_seq) {
        set_error("generate: %d cached + %d prompt + %d predicted exceed the %d-position cache", m->host_pos, n_prompt,
                  n_predict, m->s.max_seq);
        return MUYO_ESTATE;
    }
    return MUYO_OK;
}

extern "C" int muyo_model_generate_device(MuyoModel* m, const int32_t* prompt_dev, int n_prompt, int n_predict,
                                          int32_t* out_tokens_dev, void* stream)
{
    clear_error();
    int rc = check_generate(m, n_prompt, n_predict);
    if (rc)
        return rc;
    MUYO_REQUIRE(prompt_dev && (n_predict == 0 || out_tokens_dev), "generate: null buffer");
    MUYO_CUDA_TRY(cudaSetDevice(m->device));
    const cudaStream_t st = as_stream(stream);
    const int p0 = m->host_pos;
    MUYO_CUDA_TRY(cudaMemcpyAsync(m->tokens + p0, prompt_dev, sizeof(int32_t) * n_prompt, cudaMemcpyDeviceToDevice, st));
    const int total = p0 + n_prompt + n_predict;
    int fed = 0;
    if ((rc = feed_prompt(m, n_prompt, st, fed)))
        return rc;
    rc = run_steps(m, p0 + n_prompt, total, n_prompt - fed + n_predict, st);
    if (rc)
        return rc;
    if (n_predict > 0)
        MUYO_CUDA_TRY(cudaMemcpyAsync(out_tokens_dev, m->tokens + p0 + n_prompt, sizeof(int32_t) * n_predict,
                                      cudaMemcpyDeviceToDevice, st));
    return MUYO_OK;
}

extern "C" int muyo_model_generate(MuyoModel* m, const int32_t* prompt, int n_prompt, int n_predict,
                                   int32_t* out_tokens, void* stream)
{
    clear_error();
    int rc = check_generate(m, n_prompt, n_predict);
    if (rc)
        return rc;
    MUYO_REQUIRE(prompt && (n_predict == 0 || out_tokens), "generate: null buffer");
    MUYO_CUDA_TRY(cudaSetDevice(m->device));
    const cudaStream_t st = as_stream(stream);
    const int p0 = m->host_pos;
    std::memcpy(m->pinned, prompt, sizeof(int32_t) * n_prompt);
    MUYO_CUDA_TRY(cudaMemcpyAsync(m->tokens + p0, m->pinned, sizeof(int32_t) * n_prompt, cudaMemcpyHostToDevice, st));
    const int total = p0 + n_prompt + n_predict;
    int fed = 0;
    if ((rc = feed_prompt(m, n_prompt, st, fed)))
        return rc;
    rc = run_steps(m, p0 + n_prompt, total, n_prompt - fed + n_predict, st);
    if (rc)
        return rc;
    if (n_predict > 0) {
        MUYO_CUDA_TRY(cudaMemcpyAsync(m->pinned, m->tokens + p0 + n_prompt, sizeof(int32_t) * n_predict,
                                      cudaMemcpyDeviceToHost, st));
    }
    MUYO_CUDA_TRY(cudaStreamSynchronize(st));
    if (n_predict > 0)
        std::memcpy(out_tokens, m->pinned, sizeof(int32_t) * n_predict);
    return check_device_error(m, st);
}

extern "C" int muyo_model_step(MuyoModel* m, int32_t token, float* logits, int32_t* next_token, void* stream)
{
    clear_error();
    int rc = check_generate(m, 1, 0);
    if (rc)
        return rc;
    MUYO_REQUIRE(token >= 0 && token < m->s.vocab, "step: token %d outside [0, %d)", token, m->s.vocab);
    MUYO_CUDA_TRY(cudaSetDevice(m->device));
    const cudaStream_t st = as_stream(stream);
    const int p0 = m->host_pos;
    m->pinned[0] = token;
    MUYO_CUDA_TRY(cudaMemcpyAsync(m->tokens + p0, m->pinned, sizeof(int32_t), cudaMemcpyHostToDevice, st));
    rc = run_steps(m, p0 + 1, p0 + 1, 1, st);
    if (rc)
        return rc;
    if (logits)
        MUYO_CUDA_TRY(cudaMemcpyAsync(logits, m->logits, sizeof(float) * m->s.vocab, cudaMemcpyDefault, st));
    MUYO_CUDA_TRY(cudaMemcpyAsync(m->pinned + 1, &m->ctrl->greedy, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    MUYO_CUDA_TRY(cudaStreamSynchronize(st));
    if (next_token)
        *next_token = m->pinned[1];
    return check_device_error(m, st);
}

extern "C" int muyo_model_position(const MuyoModel* m, int32_t* pos)
{
    clear_error();
    MUYO_REQUIRE(m && pos, "position: null argument");
    *pos = m->host_pos;
    return MUYO_OK;
}

extern "C" int muyo_model_buffer(MuyoModel* m, const char* name, void** ptr, size_t* bytes)
{
    clear_error();
    MUYO_REQUIRE(m && name && ptr, "buffer: null argument");
    const std::string n(name);
    size_t b = 0;
    if (n == "logits") {
        *ptr = m->logits;
        b = sizeof(float) * m->s.vocab;
    } else if (n == "hidden") {
        *ptr = m->h;
        b = sizeof(float) * m->s.hidden;
    } else if (n == "k_cache") {
        *ptr = m->kc;
        b = m->kv_layer_bytes * m->s.layers;
    } else if (n == "v_cache") {
        *ptr = m->vc;
        b = m->kv_layer_bytes * m->s.layers;
    } else if (n == "tokens") {
        *ptr = m->tokens;
        b = sizeof(int32_t) * m->s.max_seq;
    } else {
        MUYO_REQUIRE(false, "buffer: unknown buffer %s", name);
    }
    if (bytes)
        *bytes = b;
    return MUYO_OK;
}

extern "C" int muyo_model_destroy(MuyoModel* m)
{
    clear_error();
    if (m) {
        cudaSetDevice(m->device);
        cudaDeviceSynchronize();
        free_model(m);
    }
    return MUYO_OK;
}

extern "C" int muyo_model_set_sampler(MuyoModel* m, const MuyoSamplerParams* p, void* stream)
{
    clear_error();
    MUYO_REQUIRE(m, "set_sampler: null model");
    MUYO_CUDA_TRY(cudaSetDevice(m->device));
    // temperature <= 0 with no penalty is the reference's plain greedy pick, which the LM head makes.
    const bool on = p && (p->temperature > 0.0f || p->repeat_penalty != 1.0f);
    if (on) {
        int rc = sample_check(p, (uint32_t)m->s.vocab, m->s.max_seq);
        if (rc)
            return rc;
        if (!m->rng)
            MUYO_CUDA_TRY(cudaMalloc(&m->rng, (muyo_sampler_state_bytes() + 15) / 16 * 16 + 16));
        const cudaStream_t st = as_stream(stream);
        rc = muyo_sampler_seed(m->rng, p->seed, st);
        if (rc)
            return rc;
        MUYO_CUDA_TRY(cudaStreamSynchronize(st));
        m->sp = *p;
    }
    const bool rerecord = m->finalized && (on || m->sampling);
    m->sampling = on;
    return rerecord ? record_graph(m) : MUYO_OK;
}

extern "C" int muyo_model_set_option(MuyoModel* m, const char* key, int value)
{
    clear_error();
    MUYO_REQUIRE(m && key, "set_option: null argument");
    const std::string k(key);
    if (k == "engine") {
        MUYO_REQUIRE(value == 0 || value == 1, "set_option: engine must be 0 (persistent) or 1 (graph)");
        m->engine = value;
        return MUYO_OK;
    }
    if (k == "prefetch") {
        MUYO_REQUIRE(value == 0 || value == 1, "set_option: prefetch must be 0 or 1");
        MUYO_REQUIRE(!m->exec, "set_option: prefetch must be set before muyo_model_finalize");
        m->prefetch_ahead = value != 0;
        return MUYO_OK;
    }
    if (k == "smem_weights") {
        MUYO_REQUIRE(value == 0 || value == 1, "set_option: smem_weights must be 0 or 1");
        MUYO_REQUIRE(!m->exec, "set_option: smem_weights must be set before muyo_model_finalize");
        m->sw = value != 0;
        return MUYO_OK;
    }
    if (k == "prefill") {
        MUYO_REQUIRE(value == 0 || value == 1, "set_option: prefill must be 0 or 1");
        MUYO_CUDA_TRY(cudaSetDevice(m->device));
        if (value) {
            const int rc = pf_alloc(m);
            if (rc)
                return rc;
        }
        m->prefill = value != 0;
        return MUYO_OK;
    }
    if (k == "prefill_positions") {
        MUYO_REQUIRE(value >= 128 && value <= kPfCapMax && value % 128 == 0,
                     "set_option: prefill_positions must be a multiple of 128 in [128, %d]", kPfCapMax);
        if (m->pf_buf) {
            set_error("set_option: prefill_positions must be set before prefill is enabled");
            return MUYO_ESTATE;
        }
        m->pf_cap = value;
        return MUYO_OK;
    }
    if (k == "prefill_tc") {
        MUYO_REQUIRE(value >= 0 && value <= 2, "set_option: prefill_tc must be 0, 1 or 2");
        m->pf_tc = value;
        return MUYO_OK;
    }
    if (k == "pdl") {
        MUYO_REQUIRE(value == 0 || value == 1, "set_option: pdl must be 0 or 1");
        MUYO_REQUIRE(!m->exec, "set_option: pdl must be set before muyo_model_finalize");
        m->pdl = value != 0;
        return MUYO_OK;
    }
    MUYO_REQUIRE(false, "set_option: unknown option %s", key);
    return MUYO_EINVAL;
}

// ---- op level: batched F16 GEMM (the prefill's projection) -----------------------------------------

extern "C" size_t muyo_cuda_mat_mul_f16_workspace_size(const MuyoMatMulParams* p)
{
    if (!p)
        return 0;
    const size_t halves = 2 * (size_t)p->tokens * (((size_t)p->ncols + 7) / 8 * 8);
    const int S = std::max(pf_splits((int)p->rows, (int)p->ncols, (int)p->tokens, true),
                           pf_splits((int)p->rows, (int)p->ncols, (int)p->tokens, false));
    const size_t part = (size_t)S * p->tokens * p->rows;
    return halves * sizeof(__half) + 256 + part * sizeof(float);
}

extern "C" int muyo_cuda_mat_mul_f16(const MuyoMatMulParams* p, const void* a, const float* x, float* y,
                                     const float* bias, void* workspace, size_t workspace_bytes, void* stream)
{
    clear_error();
    MUYO_REQUIRE(p && a && x && y, "mat_mul: null parameter block or buffer");
    const int K = (int)p->ncols, N = (int)p->rows, T = (int)p->tokens;
    const int ldx = p->stride_x ? (int)p->stride_x : K, ldy = p->stride_y ? (int)p->stride_y : N;
    MUYO_REQUIRE(K > 0 && N > 0 && T > 0, "mat_mul: ncols, rows and tokens must be positive");
    MUYO_REQUIRE(K % 8 == 0, "mat_mul: ncols %d must be a multiple of 8", K);
    MUYO_REQUIRE(ldx >= K && ldx % 4 == 0 && ldy >= N, "mat_mul: strides too small or x stride not a multiple of 4");
    MUYO_REQUIRE((p->flags & ~(MUYO_MATMUL_BIAS | MUYO_MATMUL_ACCUMULATE | MUYO_MATMUL_TCGEN05)) == 0 &&
                     (p->flags & (MUYO_MATMUL_BIAS | MUYO_MATMUL_ACCUMULATE)) != (MUYO_MATMUL_BIAS | MUYO_MATMUL_ACCUMULATE),
                 "mat_mul: flags are BIAS or ACCUMULATE");
    MUYO_REQUIRE(!(p->flags & MUYO_MATMUL_BIAS) || bias, "mat_mul: BIAS without a bias vector");
    MUYO_REQUIRE(aligned16(a) && aligned16(x), "mat_mul: a and x must be 16-byte aligned");
    MUYO_REQUIRE(workspace && workspace_bytes >= muyo_cuda_mat_mul_f16_workspace_size(p) && aligned16(workspace),
                 "mat_mul: workspace of muyo_cuda_mat_mul_f16_workspace_size bytes, 16-byte aligned, required");
    const cudaStream_t st = as_stream(stream);
    const int ldh = (K + 7) / 8 * 8;
    __half* hi = static_cast<__half*>(workspace);
    __half* lo = hi + (size_t)T * ldh;
    const size_t part_off = ((size_t)2 * T * ldh * sizeof(__half) + 255) / 256 * 256;
    float* part = reinterpret_cast<float*>(static_cast<char*>(workspace) + part_off);
    const size_t part_floats = (workspace_bytes - part_off) / sizeof(float);
    for (auto k : {k_pf_gemm<PF_STORE>, k_pf_gemm<PF_BIAS>, k_pf_gemm<PF_ADD>})
        MUYO_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPfGemmSmem));
    for (auto k : {k_pf_gemm_tc<PF_STORE>, k_pf_gemm_tc<PF_BIAS>, k_pf_gemm_tc<PF_ADD>})
        MUYO_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem));
    MUYO_CUDA_TRY(launch_kernel(k_pf_split, dim3(T), dim3(256), 0, st, true, x, ldx, K, hi, lo, ldh));
    const __half* w = static_cast<const __half*>(a);
    PfMaps maps;
    const PfMaps* tc = nullptr;
    int rc;
    if (p->flags & MUYO_MATMUL_TCGEN05) {
        if ((rc = make_map(&maps.w0, w, K, N, K, kTcBM)) || (rc = make_map(&maps.xhi, hi, K, T, ldh, kTcBN)) ||
            (rc = make_map(&maps.xlo, lo, K, T, ldh, kTcBN)))
            return rc;
        maps.w1 = maps.w0;
        tc = &maps;
    }
    if (p->flags & MUYO_MATMUL_BIAS)
        rc = pf_gemm<PF_BIAS>(w, nullptr, N, N, K, T, hi, lo, ldh, y, ldy, bias, part, part_floats, st, tc);
    else if (p->flags & MUYO_MATMUL_ACCUMULATE)
        rc = pf_gemm<PF_ADD>(w, nullptr, N, N, K, T, hi, lo, ldh, y, ldy, nullptr, part, part_floats, st, tc);
    else
        rc = pf_gemm<PF_STORE>(w, nullptr, N, N, K, T, hi, lo, ldh, y, ldy, nullptr, part, part_floats, st, tc);
    if (rc)
        return rc;
    MUYO_LAUNCH_CHECK();
    return MUYO_OK;
}
