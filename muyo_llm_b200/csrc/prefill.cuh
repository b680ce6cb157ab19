// Batched prefill: the prompt's positions go through each layer together instead of one decode
// step per token (the reference feeds a prompt one position at a time, src/FullModel.cpp:1096-1108,
// 1174-1181; its unused batched GEMM shader is shaders/llama/mul_mm.comp). The positions' keys and
// values land in the same KV cache the decode step reads; the decode step then takes over at the
// prompt's last position.
//
// Per layer, for T positions:
//   k_pf_norm_split   RMSNorm of the residual rows (the decode prologue's arithmetic and thread
//                     layout, so each row's value is bit-identical), written as two F16 halves
//   k_pf_gemm<BIAS>   QKV projection + bias
//   k_pf_rope_append  RoPE (float64 angles, as the decode step) on q and k; k and v into the cache
//   k_pf_attention    causal GQA over the cache, one CTA per (kv head, position) (F32 cache)
//   k_pf_flash        the same on the tensor cores for an F16 cache (flash attention, mma.sync)
//   k_pf_split        attention rows -> two F16 halves
//   k_pf_gemm<ADD>    O projection added to the residual
//   k_pf_norm_split, k_pf_gemm<STORE> (gate | up, two matrices in one launch), k_pf_swiglu_split,
//   k_pf_gemm<ADD>    the MLP
//
// The GEMM is weight-read bound for prompts of up to a few hundred positions (2 flops per weight
// byte per position), so by default it uses the warp-level mma.sync m16n8k16 (F16 x F16 -> F32) on
// tiles staged by cp.async; k_pf_gemm_tc is the same GEMM on tcgen05 (tensor-memory accumulator).
// An activation x enters as hi = f16(x) and lo = f16(x - hi), two products into one F32
// accumulator, which keeps the product error near F32's (2^-22 relative to |x|).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include "attention.cuh"
#include "common.cuh"

namespace muyo {

constexpr int kPfBM = 64;  // feature rows per CTA (4 warps x 16)
constexpr int kPfBN = 64;  // positions per CTA
constexpr int kPfBK = 64;  // reduction chunk per pipeline stage
constexpr int kPfLD = kPfBK + 8;  // padded row (144 bytes): ldmatrix rows fall in distinct banks
constexpr int kPfStages = 3;
constexpr int kPfThreads = 128;
constexpr int kPfStageHalfs = 3 * 64 * kPfLD;  // W tile, x-hi tile, x-lo tile
constexpr size_t kPfGemmSmem = (size_t)kPfStages * kPfStageHalfs * sizeof(__half);

enum PfEpi { PF_STORE = 0, PF_BIAS = 1, PF_ADD = 2 };

// y[t][n] (= | += | = b[n] +) sum_k W[n][k] * x[t][k] for n < N, t < T. W rows are K halves apart;
// rows [0, n_split) come from w0 and rows [n_split, N) from w1 (row n - n_split).
struct PfGemm {
    const __half* w0;
    const __half* w1;
    int n_split;
    int N, K, T;
    const __half* xhi;  // [T][ldx]
    const __half* xlo;
    int ldx;
    float* y;  // [T][ldy]
    int ldy;
    const float* bias;
};

__device__ __forceinline__ void cp_async16(unsigned dst, const void* src, bool full)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(full ? 16 : 0));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait()
{
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void ldsm_x4(unsigned addr, unsigned& r0, unsigned& r1, unsigned& r2, unsigned& r3)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// d += a (16x16, row-major) * b (16x8, k-major per column), F16 inputs, F32 accumulation.
__device__ __forceinline__ void mma_16816(float (&d)[4], unsigned a0, unsigned a1, unsigned a2, unsigned a3,
                                          unsigned b0, unsigned b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One CTA: 64 feature rows x 64 positions. Warp w owns rows [16w, 16w + 16) of the tile and all 64
// positions (8 accumulator fragments of 16 x 8). K advances 64 at a time through a 3-stage cp.async
// ring; chunks past N, T or K are zero-filled (K is a multiple of 8). With gridDim.z = S > 1 the CTA
// covers the z-th of S contiguous ranges of K stages and stores its raw sums to part[z][t][n]
// (k_pf_reduce adds the S ranges in order and applies the epilogue).
template <int EPI>
__global__ void __launch_bounds__(kPfThreads, 2) k_pf_gemm(PfGemm g, float* part)
{
    extern __shared__ __align__(16) __half pf_smem[];
    pdl_wait();
    pdl_trigger();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n0 = blockIdx.x * kPfBM, t0 = blockIdx.y * kPfBN;
    const int nk_all = (g.K + kPfBK - 1) / kPfBK, S = gridDim.z, z = blockIdx.z;
    const int kt0 = (int)((long long)nk_all * z / S), kt1 = (int)((long long)nk_all * (z + 1) / S);
    const int nk = kt1 - kt0;
    const unsigned sbase = (unsigned)__cvta_generic_to_shared(pf_smem);

    // This thread's 12 chunks of a stage (3 tiles x 64 rows x 8 chunks over 128 threads): chunk
    // c = tid + 128 i is tile i / 4, row (c >> 3) & 63, 16-byte column c & 7; its source row is fixed.
    const __half* src_row[12];
    bool row_ok[12];
    unsigned dst_off[12];
    int kcol[12];
#pragma unroll
    for (int i = 0; i < 12; ++i) {
        const int c = tid + i * kPfThreads, tile = i >> 2, r = (c >> 3) & 63, ch = c & 7;
        dst_off[i] = (unsigned)((tile * 64 * kPfLD + r * kPfLD + ch * 8) * 2);
        kcol[i] = ch * 8;
        if (tile == 0) {
            const int n = n0 + r;
            row_ok[i] = n < g.N;
            src_row[i] = !row_ok[i] ? g.w0 : (n < g.n_split ? g.w0 + (size_t)n * g.K : g.w1 + (size_t)(n - g.n_split) * g.K);
        } else {
            const int t = t0 + r;
            const __half* xb = tile == 1 ? g.xhi : g.xlo;
            row_ok[i] = t < g.T;
            src_row[i] = row_ok[i] ? xb + (size_t)t * g.ldx : xb;
        }
    }
    auto load_stage = [&](int buf, int kt) {
        const int k0 = kt * kPfBK;
        const unsigned st = sbase + (unsigned)(buf * kPfStageHalfs * 2);
#pragma unroll
        for (int i = 0; i < 12; ++i) {
            const int k = k0 + kcol[i];
            const bool ok = row_ok[i] && k < g.K;
            cp_async16(st + dst_off[i], ok ? src_row[i] + k : src_row[i], ok);
        }
    };

    float acc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e)
            acc[j][e] = 0.0f;
#pragma unroll
    for (int s = 0; s < kPfStages - 1; ++s) {
        if (s < nk)
            load_stage(s, kt0 + s);
        cp_async_commit();
    }
    const int mat = lane >> 3;
    for (int i = 0; i < nk; ++i) {
        cp_async_wait<kPfStages - 2>();
        __syncthreads();  // stage i is visible, and every warp is done with the buffer refilled next
        {
            const int nxt = i + kPfStages - 1;
            if (nxt < nk)
                load_stage(nxt % kPfStages, kt0 + nxt);
            cp_async_commit();
        }
        const unsigned ws = sbase + (unsigned)((i % kPfStages) * kPfStageHalfs * 2);
        const unsigned xh = ws + 64 * kPfLD * 2, xl = ws + 2 * 64 * kPfLD * 2;
#pragma unroll
        for (int kk = 0; kk < kPfBK; kk += 16) {
            unsigned a0, a1, a2, a3;
            {  // matrices: rows 0-7 / 8-15 x k 0-7 / 8-15 of the warp's 16 rows -> a0..a3
                const int r = warp * 16 + (mat & 1) * 8 + (lane & 7), c = kk + (mat >> 1) * 8;
                ldsm_x4(ws + (unsigned)((r * kPfLD + c) * 2), a0, a1, a2, a3);
            }
            unsigned bh[8][2], bl[8][2];
#pragma unroll
            for (int j2 = 0; j2 < 4; ++j2) {  // positions 16*j2 .. +15: two 8-wide fragments
                const int r = j2 * 16 + (mat >> 1) * 8 + (lane & 7), c = kk + (mat & 1) * 8;
                ldsm_x4(xh + (unsigned)((r * kPfLD + c) * 2), bh[2 * j2][0], bh[2 * j2][1], bh[2 * j2 + 1][0],
                        bh[2 * j2 + 1][1]);
                ldsm_x4(xl + (unsigned)((r * kPfLD + c) * 2), bl[2 * j2][0], bl[2 * j2][1], bl[2 * j2 + 1][0],
                        bl[2 * j2 + 1][1]);
            }
            // eight independent accumulators between two products into the same one
#pragma unroll
            for (int j = 0; j < 8; ++j)
                mma_16816(acc[j], a0, a1, a2, a3, bh[j][0], bh[j][1]);
#pragma unroll
            for (int j = 0; j < 8; ++j)
                mma_16816(acc[j], a0, a1, a2, a3, bl[j][0], bl[j][1]);
        }
    }
    cp_async_wait<0>();
    // fragment (j, e): feature row 16w + lane/4 (+8 for e >= 2), position 8j + 2*(lane%4) + (e & 1)
    const int gr = lane >> 2, tq = lane & 3;
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int n = n0 + warp * 16 + gr + (e >> 1) * 8;
            const int t = t0 + j * 8 + tq * 2 + (e & 1);
            if (n < g.N && t < g.T) {
                if (S > 1) {
                    part[((size_t)z * g.T + t) * g.N + n] = acc[j][e];
                } else {
                    float* yp = g.y + (size_t)t * g.ldy + n;
                    float v = acc[j][e];
                    if (EPI == PF_BIAS)
                        v = v + g.bias[n];
                    if (EPI == PF_ADD)
                        v = *yp + v;
                    *yp = v;
                }
            }
        }
}

// y[t][n] = epilogue(part[0][t][n] + part[1][t][n] + ... + part[S-1][t][n]), left to right.
template <int EPI>
__global__ void __launch_bounds__(256) k_pf_reduce(PfGemm g, const float* __restrict__ part, int S)
{
    pdl_wait();
    pdl_trigger();
    const size_t total = (size_t)g.T * g.N;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / g.N), n = (int)(i % g.N);
        float v = part[i];
        for (int z = 1; z < S; ++z)
            v += part[(size_t)z * total + i];
        float* yp = g.y + (size_t)t * g.ldy + n;
        if (EPI == PF_BIAS)
            v = v + g.bias[n];
        if (EPI == PF_ADD)
            v = *yp + v;
        *yp = v;
    }
}

// ---- the same GEMM on the 5th-generation tensor cores (tcgen05), fed by TMA -------------------------
// Persistent CTAs (one per SM) over work items = (128-feature tile, 128-position tile, K range);
// 6 warps with fixed roles:
//   warp 4, one lane: the producer. Per 64-deep K stage it arms the stage's `full` mbarrier with the
//     stage's 48 KB and issues 24 two-dimensional TMA tile loads (8 K-chunks of 8 halves for each of
//     W, x-hi and x-lo), waiting on the stage's `empty` barrier once the 4-stage ring wraps; it runs
//     ahead across work items;
//   warp 5: allocates 256 tensor-memory columns (two 128-column F32 accumulators); its lane 0 is the
//     MMA issuer: it waits on `full`, issues 4 K-steps x 2 MMAs (x-hi, x-lo) of 128 x 128 x 16, and
//     commits each stage to `empty`; at the end of a work item it commits the accumulator to
//     `acc_full` (after waiting on `acc_empty` before reusing a buffer);
//   warps 0-3: the epilogue. Warp w reads accumulator lanes 32w .. 32w + 31 (tcgen05.ld 32x32b),
//     stores, and arrives on `acc_empty`; the MMA issuer meanwhile fills the other accumulator.
// Each operand tile of a stage is ONE TMA box of 64 halves x 128 rows (16 KB) with the 128-byte
// swizzle: row r's 128 bytes sit at r * 128 with their 16-byte chunks permuted by r mod 8, the
// canonical K-major SWIZZLE_128B layout. The UMMA descriptors name that layout (stride-byte offset
// 1024 between 8-row groups); K-step k of the 64-deep stage starts 32 * k bytes into the tile, and
// the hardware applies the same permutation to the advanced address (tiles are 1 KB-aligned). Rows
// and columns outside the tensors are zero-filled by the TMA. Every wait is bounded (2 s): on expiry
// the error word gets 6, the roles stop, and the CTA still frees its TMEM.
constexpr int kTcBM = 128, kTcBN = 128, kTcBK = 64, kTcStages = 4, kTcThreads = 192;
constexpr int kTcWBytes = kTcBM * kTcBK * 2;               // 16 KB
constexpr int kTcXBytes = kTcBN * kTcBK * 2;               // 16 KB
constexpr int kTcStageBytes = kTcWBytes + 2 * kTcXBytes;   // 48 KB
constexpr size_t kTcSmem = (size_t)kTcStages * kTcStageBytes + 1024;  // + alignment slack
constexpr int kTcTmemCols = 2 * kTcBN;                     // two accumulators

// UMMA shared-memory descriptor of a K-major SWIZZLE_128B tile: start >> 4 in [0,14), leading-byte
// offset in [16,30) (unused by swizzled K-major layouts; 1), stride-byte offset 1024 >> 4 in
// [32,46), version 1 in [46,48), base offset 0 in [49,52) (1 KB-aligned tiles), layout 2 (128-byte
// swizzle) in [61,64).
__device__ __forceinline__ uint64_t umma_desc_sw128(unsigned saddr)
{
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}

// Instruction descriptor, kind::f16: F32 accumulator (bits [4,6) = 1), A and B F16 (0), both
// K-major, N >> 3 in [17,23), M >> 4 in [24,29).
constexpr uint32_t kTcIdesc = (1u << 4) | ((uint32_t)(kTcBN >> 3) << 17) | ((uint32_t)(kTcBM >> 4) << 24);

__device__ __forceinline__ void tc_mma(uint32_t tmem, uint64_t da, uint64_t db, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem),
        "l"(da), "l"(db), "r"(kTcIdesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// 32 consecutive accumulator columns of this warp's 32 lanes: thread l of warp w gets row 32w + l.
__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

// Bounded wait for `parity` of `bar`; false (error word 6) on expiry.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, unsigned parity, int* err)
{
    if (mbar_try_wait(bar, parity))
        return true;
    const unsigned long long t0 = now_ns();
    while (!mbar_try_wait(bar, parity))
        if (now_ns() - t0 > kWaitLimitNs) {
            if (err)
                atomicMax(err, 6);
            return false;
        }
    return true;
}

// 2-D TMA tile load into this CTA's shared memory, completing on `bar` (no multicast).
__device__ __forceinline__ void tma_load_2d(unsigned dst, const void* map, int x, int y, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// The tile's W rows come from tw0 or, past n_split (a multiple of 128), from tw1 (row n - n_split).
template <int EPI>
__global__ void __launch_bounds__(kTcThreads, 1)
    k_pf_gemm_tc(PfGemm g, float* part, int* err, int S, const __grid_constant__ CUtensorMap tw0,
                 const __grid_constant__ CUtensorMap tw1, const __grid_constant__ CUtensorMap txh,
                 const __grid_constant__ CUtensorMap txl)
{
    extern __shared__ unsigned char tc_raw[];
    __shared__ __align__(8) uint64_t full_bar[kTcStages];
    __shared__ __align__(8) uint64_t empty_bar[kTcStages];
    __shared__ __align__(8) uint64_t acc_full[2];
    __shared__ __align__(8) uint64_t acc_empty[2];
    __shared__ uint32_t tmem_base;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (warp == 5) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                     "r"(kTcTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], 128);  // every epilogue thread arrives
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    pdl_wait();  // x comes from the previous kernel: no TMA load before this point
    pdl_trigger();
    const unsigned sbase = (smem_u32(tc_raw) + 1023u) & ~1023u;  // 1 KB-aligned ring
    const int ntn = (g.N + kTcBM - 1) / kTcBM, ntt = (g.T + kTcBN - 1) / kTcBN;  // S: K ranges
    const int nk_all = (g.K + kTcBK - 1) / kTcBK, items = ntn * ntt * S;
    // work item -> (feature tile, position tile, K range [kt0, kt1))
    auto item_geom = [&](int it, int& n0, int& t0, int& z, int& kt0, int& kt1) {
        n0 = (it % ntn) * kTcBM;
        t0 = ((it / ntn) % ntt) * kTcBN;
        z = it / (ntn * ntt);
        kt0 = (int)((long long)nk_all * z / S);
        kt1 = (int)((long long)nk_all * (z + 1) / S);
    };

    if (warp == 4) {
        if (lane == 0) {  // producer
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tw0)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&txh)) : "memory");
            int gs = 0;  // stages issued by this CTA
            bool stop = false;
            for (int it = blockIdx.x; it < items && !stop; it += gridDim.x) {
                int n0, t0, z, kt0, kt1;
                item_geom(it, n0, t0, z, kt0, kt1);
                const CUtensorMap* tw = n0 < g.n_split ? &tw0 : &tw1;
                const int wrow = n0 < g.n_split ? n0 : n0 - g.n_split;
                for (int kt = kt0; kt < kt1; ++kt, ++gs) {
                    const int s = gs % kTcStages;
                    if (gs >= kTcStages && !tc_wait(&empty_bar[s], (unsigned)(((gs / kTcStages) - 1) & 1), err)) {
                        stop = true;
                        break;
                    }
                    mbar_expect_tx(&full_bar[s], (unsigned)kTcStageBytes);
                    const unsigned st = sbase + (unsigned)(s * kTcStageBytes);
                    const int k0 = kt * kTcBK;
                    tma_load_2d(st, tw, k0, wrow, &full_bar[s]);
                    tma_load_2d(st + (unsigned)kTcWBytes, &txh, k0, t0, &full_bar[s]);
                    tma_load_2d(st + (unsigned)(kTcWBytes + kTcXBytes), &txl, k0, t0, &full_bar[s]);
                }
            }
        }
    } else if (warp == 5) {
        if (lane == 0) {  // MMA issuer
            int gs = 0, j = 0;  // stages consumed, work items done by this CTA
            bool stop = false;
            for (int it = blockIdx.x; it < items && !stop; it += gridDim.x, ++j) {
                int n0, t0, z, kt0, kt1;
                item_geom(it, n0, t0, z, kt0, kt1);
                const int a = j & 1;
                if (j >= 2 && !tc_wait(&acc_empty[a], (unsigned)(((j >> 1) - 1) & 1), err))
                    break;
                tc_fence_after();
                const uint32_t acc = tmem + (uint32_t)(a * kTcBN);
                for (int kt = kt0; kt < kt1; ++kt, ++gs) {
                    const int s = gs % kTcStages;
                    if (!tc_wait(&full_bar[s], (unsigned)((gs / kTcStages) & 1), err)) {
                        stop = true;
                        break;
                    }
                    tc_fence_after();
                    const unsigned st = sbase + (unsigned)(s * kTcStageBytes);
#pragma unroll
                    for (int k = 0; k < kTcBK / 16; ++k) {  // K-step k: bytes 32k .. 32k + 31 of each row
                        const uint64_t da = umma_desc_sw128(st + (unsigned)(32 * k));
                        const uint64_t dh = umma_desc_sw128(st + (unsigned)(kTcWBytes + 32 * k));
                        const uint64_t dl = umma_desc_sw128(st + (unsigned)(kTcWBytes + kTcXBytes + 32 * k));
                        tc_mma(acc, da, dh, (kt > kt0 || k > 0) ? 1u : 0u);
                        tc_mma(acc, da, dl, 1u);
                    }
                    tc_commit(&empty_bar[s]);
                }
                tc_commit(&acc_full[a]);  // the item's accumulator is complete once its MMAs are
            }
        }
    } else {  // epilogue: warps 0-3, warp w owns accumulator lanes (feature rows) 32w .. 32w + 31
        int j = 0;
        for (int it = blockIdx.x; it < items; it += gridDim.x, ++j) {
            int n0, t0, z, kt0, kt1;
            item_geom(it, n0, t0, z, kt0, kt1);
            const int a = j & 1;
            bool ok = true;
            if (lane == 0)
                ok = tc_wait(&acc_full[a], (unsigned)((j >> 1) & 1), err);
            ok = __shfl_sync(0xffffffffu, ok, 0);  // one decision per warp (tcgen05.ld is warp-wide)
            if (!ok)
                break;
            tc_fence_after();
            const int n = n0 + warp * 32 + lane;
#pragma unroll 1
            for (int q = 0; q < kTcBN / 32; ++q) {
                uint32_t r[32];
                tc_ld32(tmem + (uint32_t)(a * kTcBN) + ((uint32_t)(warp * 32) << 16) + (uint32_t)(q * 32), r);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (n < g.N) {
#pragma unroll
                    for (int c = 0; c < 32; ++c) {
                        const int t = t0 + q * 32 + c;
                        if (t < g.T) {
                            const float v0 = __uint_as_float(r[c]);
                            if (S > 1) {
                                part[((size_t)z * g.T + t) * g.N + n] = v0;
                            } else {
                                float* yp = g.y + (size_t)t * g.ldy + n;
                                float v = v0;
                                if (EPI == PF_BIAS)
                                    v = v + g.bias[n];
                                if (EPI == PF_ADD)
                                    v = *yp + v;
                                *yp = v;
                            }
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[a]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols) : "memory");
    }
}

__device__ __forceinline__ void split_store(__half* hi, __half* lo, float4 v)
{
    const __half2 h01 = __floats2half2_rn(v.x, v.y), h23 = __floats2half2_rn(v.z, v.w);
    const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
    const __half2 l01 = __floats2half2_rn(v.x - f01.x, v.y - f01.y), l23 = __floats2half2_rn(v.z - f23.x, v.w - f23.y);
    reinterpret_cast<__half2*>(hi)[0] = h01;
    reinterpret_cast<__half2*>(hi)[1] = h23;
    reinterpret_cast<__half2*>(lo)[0] = l01;
    reinterpret_cast<__half2*>(lo)[1] = l23;
}

// Row t of x [T][ldx] (F32) -> hi/lo [T][ldh]; K a multiple of 4, rows 16-byte aligned.
__global__ void __launch_bounds__(256) k_pf_split(const float* __restrict__ x, int ldx, int K, __half* hi, __half* lo,
                                                  int ldh)
{
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x;
    for (int q = threadIdx.x; q < K / 4; q += blockDim.x) {
        const float4 v = reinterpret_cast<const float4*>(x + (size_t)t * ldx)[q];
        split_store(hi + (size_t)t * ldh + 4 * q, lo + (size_t)t * ldh + 4 * q, v);
    }
}

// RMSNorm of row t (x / sqrt(mean(x^2) + eps) * w) -> hi/lo. 256 threads, each adding the squares
// of the float4s q = tid + 256 j in that order, then block_sum: the decode prologue's arithmetic.
__global__ void __launch_bounds__(256) k_pf_norm_split(const float* __restrict__ x, int ldx,
                                                       const float* __restrict__ w, float eps, int K, __half* hi,
                                                       __half* lo, int ldh)
{
    __shared__ float red[32];
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x, tid = threadIdx.x, Q = K / 4;
    const float4* x4 = reinterpret_cast<const float4*>(x + (size_t)t * ldx);
    float ss = 0.0f;
    for (int q = tid; q < Q; q += blockDim.x) {
        const float4 v = x4[q];
        ss = fmaf(v.x, v.x, ss);
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
    }
    ss = block_sum(ss, red);
    const float s = __fsqrt_rn(__fdiv_rn(ss, (float)K) + eps);
    const float4* w4 = reinterpret_cast<const float4*>(w);
    for (int q = tid; q < Q; q += blockDim.x) {
        const float4 v = x4[q], ww = w4[q];
        const float4 y = make_float4(__fdiv_rn(v.x, s) * ww.x, __fdiv_rn(v.y, s) * ww.y, __fdiv_rn(v.z, s) * ww.z,
                                     __fdiv_rn(v.w, s) * ww.w);
        split_store(hi + (size_t)t * ldh + 4 * q, lo + (size_t)t * ldh + 4 * q, y);
    }
}

// act = silu(gate) * up for row t of gu [T][2F] (gate | up) -> hi/lo [T][ldh].
__global__ void __launch_bounds__(256) k_pf_swiglu_split(const float* __restrict__ gu, int F, __half* hi, __half* lo,
                                                         int ldh)
{
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x;
    const float4* g4 = reinterpret_cast<const float4*>(gu + (size_t)t * 2 * F);
    const float4* u4 = reinterpret_cast<const float4*>(gu + (size_t)t * 2 * F + F);
    for (int q = threadIdx.x; q < F / 4; q += blockDim.x) {
        const float4 gv = g4[q], uv = u4[q];
        const float4 a = make_float4(silu_mul(gv.x, uv.x), silu_mul(gv.y, uv.y), silu_mul(gv.z, uv.z),
                                     silu_mul(gv.w, uv.w));
        split_store(hi + (size_t)t * ldh + 4 * q, lo + (size_t)t * ldh + 4 * q, a);
    }
}

// x[t][:] = embedding row of tokens[t] (F16 -> F32); an id outside [0, vocab) gathers row 0, as the
// decode step does.
__global__ void __launch_bounds__(256) k_pf_embed(const __half* __restrict__ embd, const int32_t* tokens, int vocab,
                                                  int H, float* x)
{
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x;
    int tok = tokens[t];
    if (tok < 0 || tok >= vocab)
        tok = 0;
    const __half* row = embd + (size_t)tok * H;
    for (int k = threadIdx.x; k < H; k += blockDim.x)
        x[(size_t)t * H + k] = __half2float(row[k]);
}

struct PfRope {
    const float* qkv;  // [T][ldqkv]: q (heads*HD) | k (kv_heads*HD) | v (kv_heads*HD)
    int ldqkv;
    float* q;  // [T][heads*HD], rotated
    int p0, heads, kv_heads, max_seq;
    const double* cs;  // [max_seq][HD] cos | sin
};

// Block (t, h): q head h < heads is rotated into q; kv head h - heads has its key rotated and its
// key and value written at position p0 + t of the cache (the decode step's rounding to KV).
template <typename KV, int HD>
__global__ void __launch_bounds__(HD) k_pf_rope_append(PfRope r, KV* kc, KV* vc)
{
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x, h = blockIdx.y, j = threadIdx.x, pos = r.p0 + t;
    const float* row = r.qkv + (size_t)t * r.ldqkv;
    const double c = j < HD / 2 ? __ldg(r.cs + (size_t)pos * HD + j) : 0.0;
    const double s = j < HD / 2 ? __ldg(r.cs + (size_t)pos * HD + HD / 2 + j) : 0.0;
    if (h < r.heads) {
        if (j < HD / 2) {
            const float* src = row + h * HD;
            float y0, y1;
            rope_pair_f64(src[j], src[j + HD / 2], c, s, y0, y1);
            float* dst = r.q + (size_t)t * r.heads * HD + h * HD;
            dst[j] = y0;
            dst[j + HD / 2] = y1;
        }
        return;
    }
    const int kh = h - r.heads;
    const size_t at = ((size_t)kh * r.max_seq + pos) * HD;
    if (j < HD / 2) {
        const float* src = row + (r.heads + kh) * HD;
        float y0, y1;
        rope_pair_f64(src[j], src[j + HD / 2], c, s, y0, y1);
        kc[at + j] = kv_round<KV>(y0);
        kc[at + j + HD / 2] = kv_round<KV>(y1);
    }
    vc[at + j] = kv_round<KV>(row[(r.heads + r.kv_heads + kh) * HD + j]);
}

struct PfAttn {
    const float* q;  // [T][heads*HD], rotated
    float* out;      // [T][heads*HD]
    int p0, heads, kv_heads, gqa, max_seq;
    float scale;
};

constexpr int kPfAttnKeys = 64;
constexpr int kPfAttnThreads = 256;

// CTA (kv head kh, position t): the gqa query heads of kh at position pos = p0 + t attend to keys
// 0..pos of the cache. Keys go through shared memory 64 at a time with an online softmax (running
// max m, sum l, output o rescaled by exp(m_old - m_new)); scores, exponentials and the P.V products
// are formed as in the decode step's attention.
template <typename KV, int HD>
__global__ void __launch_bounds__(kPfAttnThreads) k_pf_attention(PfAttn a, const KV* __restrict__ kc,
                                                                  const KV* __restrict__ vc)
{
    constexpr int LD = HD + 1;
    extern __shared__ float pa_smem[];
    const int G = a.gqa;
    float* Ks = pa_smem;                   // [64][LD]
    float* Vs = Ks + kPfAttnKeys * LD;     // [64][LD]
    float* Qs = Vs + kPfAttnKeys * LD;     // [G][HD]
    float* Os = Qs + G * HD;               // [G][HD]
    float* Ps = Os + G * HD;               // [G][64]
    float* Ms = Ps + G * kPfAttnKeys;      // [G] running max
    float* Ls = Ms + G;                    // [G] running sum
    float* As = Ls + G;                    // [G] rescale of this chunk
    pdl_wait();
    pdl_trigger();
    const int kh = blockIdx.x, t = blockIdx.y, tid = threadIdx.x, nt = blockDim.x;
    const int pos = a.p0 + t, n = pos + 1;
    const size_t head_base = (size_t)kh * a.max_seq * HD;
    for (int e = tid; e < G * HD; e += nt) {
        Qs[e] = a.q[(size_t)t * a.heads * HD + (size_t)kh * G * HD + e];
        Os[e] = 0.0f;
    }
    if (tid < G) {
        Ms[tid] = -INFINITY;
        Ls[tid] = 0.0f;
    }
    for (int key0 = 0; key0 < n; key0 += kPfAttnKeys) {
        const int nk = min(kPfAttnKeys, n - key0);
        __syncthreads();  // the previous chunk's readers are done
        for (int e = tid; e < nk * HD; e += nt) {
            const int r = e / HD, d = e % HD;
            const size_t off = head_base + (size_t)(key0 + r) * HD + d;
            Ks[r * LD + d] = kv_value<KV>(kc[off]);
            Vs[r * LD + d] = kv_value<KV>(vc[off]);
        }
        __syncthreads();
        {
            const int kt = tid % kPfAttnKeys, h0 = tid / kPfAttnKeys, hs = nt / kPfAttnKeys;
            for (int gq = h0; gq < G; gq += hs) {
                float sc = -INFINITY;
                if (kt < nk) {
                    float dot = 0.0f;
#pragma unroll 16
                    for (int d = 0; d < HD; ++d)
                        dot = fmaf(Qs[gq * HD + d], Ks[kt * LD + d], dot);
                    sc = dot * a.scale;
                }
                Ps[gq * kPfAttnKeys + kt] = sc;
            }
        }
        __syncthreads();
        {
            const int lane = tid & 31, warp = tid >> 5, nw = nt / 32;
            for (int gq = warp; gq < G; gq += nw) {
                float m = -INFINITY;
                for (int k = lane; k < kPfAttnKeys; k += 32)
                    m = fmaxf(m, Ps[gq * kPfAttnKeys + k]);
                m = warp_max(m);
                const float m_old = Ms[gq], m_new = fmaxf(m_old, m);
                float l = 0.0f;
                for (int k = lane; k < kPfAttnKeys; k += 32) {
                    const float e = k < nk ? expf(Ps[gq * kPfAttnKeys + k] - m_new) : 0.0f;
                    Ps[gq * kPfAttnKeys + k] = e;
                    l += e;
                }
                l = warp_sum(l);
                if (lane == 0) {
                    const float alpha = expf(m_old - m_new);  // 0 for the first chunk (m_old = -inf)
                    As[gq] = alpha;
                    Ls[gq] = Ls[gq] * alpha + l;
                    Ms[gq] = m_new;
                }
            }
        }
        __syncthreads();
        for (int e = tid; e < G * HD; e += nt) {
            const int gq = e / HD, d = e % HD;
            float o = Os[e] * As[gq];
            for (int k = 0; k < nk; ++k)
                o = fmaf(Ps[gq * kPfAttnKeys + k], Vs[k * LD + d], o);
            Os[e] = o;
        }
    }
    __syncthreads();
    for (int e = tid; e < G * HD; e += nt) {
        const int gq = e / HD;
        a.out[(size_t)t * a.heads * HD + (size_t)kh * G * HD + e] = __fdiv_rn(Os[e], Ls[gq]);
    }
}

// ---- causal GQA attention for an F16 cache on the tensor cores (flash attention) -------------------
//
// CTA (64-position query tile, query head h): 4 warps, warp w owns query rows [16w, 16w + 16). Keys
// and values stream through shared memory 64 positions at a time (a 2-stage cp.async ring, rows
// padded to HD + 8 halves so the fragment reads are conflict-free); only the tiles at or below the
// tile's last position are read (causal). Per key tile:
//   S = Q.K^T   mma.sync m16n8k16 with Q as hi + lo F16 halves (q - f32(hi) in lo), so the scores
//               keep F32-level accuracy against the cache's exact F16 keys;
//   online softmax in registers (row max and sum across the quad of lanes that share a row);
//   O += P.V    P (exp of the scaled scores) again as hi + lo halves, V read with ldmatrix.trans.
// Keys after a query's position get exp(-inf) = 0; rows past T are computed but not stored.
// Output: O / l in F32.
constexpr int kPfFlashRows = 64, kPfFlashKeys = 64, kPfFlashThreads = 128;

__device__ __forceinline__ void ldsm_x4_t(unsigned addr, unsigned& r0, unsigned& r1, unsigned& r2, unsigned& r3)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// hi = f16(x), lo = f16(x - hi), packed as (element 0, element 1) half2 words.
__device__ __forceinline__ void split2(float x0, float x1, unsigned& hi, unsigned& lo)
{
    const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
    const __half l0 = __float2half_rn(x0 - __half2float(h0)), l1 = __float2half_rn(x1 - __half2float(h1));
    hi = (unsigned)__half_as_ushort(h0) | ((unsigned)__half_as_ushort(h1) << 16);
    lo = (unsigned)__half_as_ushort(l0) | ((unsigned)__half_as_ushort(l1) << 16);
}

template <int HD>
constexpr size_t pf_flash_smem()
{
    return (size_t)2 * 2 * kPfFlashKeys * (HD + 8) * sizeof(__half);  // 2 stages x (K, V)
}

template <int HD>
__global__ void __launch_bounds__(kPfFlashThreads) k_pf_flash(PfAttn a, int T, const __half* __restrict__ kc,
                                                              const __half* __restrict__ vc)
{
    constexpr int LDS = HD + 8;            // halves per shared-memory row (16-byte multiple)
    constexpr int KS = HD / 16;            // k-steps of Q.K^T
    constexpr int ND = HD / 8;             // 8-wide output column tiles
    constexpr int NT = kPfFlashKeys / 8;   // 8-key score tiles
    constexpr int CH = HD / 8;             // 16-byte chunks per row
    extern __shared__ __align__(16) __half pf_flash_smem_buf[];
    pdl_wait();
    pdl_trigger();
    const int tile = blockIdx.x, h = blockIdx.y, kh = h / a.gqa;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, qr = lane >> 2, qc = (lane & 3) * 2;
    const int t0 = tile * kPfFlashRows;
    const int t_last = min(t0 + kPfFlashRows, T) - 1;
    const int n_keys = a.p0 + t_last + 1;  // keys 0 .. p0 + t_last
    const size_t head_base = (size_t)kh * a.max_seq * HD;
    const unsigned sbase = smem_u32(pf_flash_smem_buf);
    constexpr unsigned kStage = 2u * kPfFlashKeys * LDS * 2u;  // bytes of one stage (K then V)

    auto load_tile = [&](int j0, int stage) {
        const unsigned kb = sbase + (unsigned)stage * kStage, vb = kb + (unsigned)(kPfFlashKeys * LDS * 2);
        for (int c = tid; c < kPfFlashKeys * CH; c += kPfFlashThreads) {
            const int r = c / CH, ch = c % CH, key = j0 + r;
            const bool ok = key < n_keys;
            const size_t off = head_base + (size_t)(ok ? key : 0) * HD + ch * 8;
            const unsigned so = (unsigned)((r * LDS + ch * 8) * 2);
            cp_async16(kb + so, kc + off, ok);
            cp_async16(vb + so, vc + off, ok);
        }
        cp_async_commit();
    };
    load_tile(0, 0);

    // Q fragments (rows r0 = t0 + 16w + qr and r0 + 8), pre-split into F16 halves.
    unsigned qh[KS][4], ql[KS][4];
    {
        const int ra = t0 + warp * 16 + qr, rb = ra + 8;
        const float* qa = a.q + (size_t)ra * a.heads * HD + (size_t)h * HD;
        const float* qb = a.q + (size_t)rb * a.heads * HD + (size_t)h * HD;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            const int c = ks * 16 + qc;
            const float2 x0 = ra < T ? *reinterpret_cast<const float2*>(qa + c) : make_float2(0.f, 0.f);
            const float2 x1 = rb < T ? *reinterpret_cast<const float2*>(qb + c) : make_float2(0.f, 0.f);
            const float2 x2 = ra < T ? *reinterpret_cast<const float2*>(qa + c + 8) : make_float2(0.f, 0.f);
            const float2 x3 = rb < T ? *reinterpret_cast<const float2*>(qb + c + 8) : make_float2(0.f, 0.f);
            split2(x0.x, x0.y, qh[ks][0], ql[ks][0]);
            split2(x1.x, x1.y, qh[ks][1], ql[ks][1]);
            split2(x2.x, x2.y, qh[ks][2], ql[ks][2]);
            split2(x3.x, x3.y, qh[ks][3], ql[ks][3]);
        }
    }
    const int pos_a = a.p0 + t0 + warp * 16 + qr, pos_b = pos_a + 8;  // query positions of this lane's rows
    float o[ND][4];
#pragma unroll
    for (int nd = 0; nd < ND; ++nd)
        o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.0f;
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.0f, l_b = 0.0f;

    const int n_tiles = (n_keys + kPfFlashKeys - 1) / kPfFlashKeys;
    for (int jt = 0; jt < n_tiles; ++jt) {
        const int j0 = jt * kPfFlashKeys, stage = jt & 1;
        if (jt + 1 < n_tiles) {
            load_tile(j0 + kPfFlashKeys, stage ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const unsigned kb = sbase + (unsigned)stage * kStage, vb = kb + (unsigned)(kPfFlashKeys * LDS * 2);
        const __half* ks_ptr = pf_flash_smem_buf + (size_t)stage * (kStage / 2);

        float sc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.0f;
            const __half* krow = ks_ptr + (nt * 8 + qr) * LDS + qc;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                const unsigned b0 = *reinterpret_cast<const unsigned*>(krow + ks * 16);
                const unsigned b1 = *reinterpret_cast<const unsigned*>(krow + ks * 16 + 8);
                mma_16816(sc[nt], qh[ks][0], qh[ks][1], qh[ks][2], qh[ks][3], b0, b1);
                mma_16816(sc[nt], ql[ks][0], ql[ks][1], ql[ks][2], ql[ks][3], b0, b1);
            }
        }
        // Scale, mask (key > query position), row maxima.
        float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int key = j0 + nt * 8 + qc;
            sc[nt][0] = key <= pos_a ? sc[nt][0] * a.scale : -INFINITY;
            sc[nt][1] = key + 1 <= pos_a ? sc[nt][1] * a.scale : -INFINITY;
            sc[nt][2] = key <= pos_b ? sc[nt][2] * a.scale : -INFINITY;
            sc[nt][3] = key + 1 <= pos_b ? sc[nt][3] * a.scale : -INFINITY;
            mx_a = fmaxf(mx_a, fmaxf(sc[nt][0], sc[nt][1]));
            mx_b = fmaxf(mx_b, fmaxf(sc[nt][2], sc[nt][3]));
        }
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
        const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
        // A row with every key so far masked keeps m = -inf; its exponentials are 0 (no NaN).
        const float base_a = mn_a == -INFINITY ? 0.0f : mn_a, base_b = mn_b == -INFINITY ? 0.0f : mn_b;
        const float al_a = expf(m_a - base_a), al_b = expf(m_b - base_b);
        m_a = mn_a, m_b = mn_b;
        float rs_a = 0.0f, rs_b = 0.0f;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            sc[nt][0] = expf(sc[nt][0] - base_a);
            sc[nt][1] = expf(sc[nt][1] - base_a);
            sc[nt][2] = expf(sc[nt][2] - base_b);
            sc[nt][3] = expf(sc[nt][3] - base_b);
            rs_a += sc[nt][0] + sc[nt][1];
            rs_b += sc[nt][2] + sc[nt][3];
        }
        rs_a += __shfl_xor_sync(0xffffffffu, rs_a, 1);
        rs_a += __shfl_xor_sync(0xffffffffu, rs_a, 2);
        rs_b += __shfl_xor_sync(0xffffffffu, rs_b, 1);
        rs_b += __shfl_xor_sync(0xffffffffu, rs_b, 2);
        l_a = l_a * al_a + rs_a;
        l_b = l_b * al_b + rs_b;
#pragma unroll
        for (int nd = 0; nd < ND; ++nd) {
            o[nd][0] *= al_a, o[nd][1] *= al_a;
            o[nd][2] *= al_b, o[nd][3] *= al_b;
        }
        // O += P.V: key step kk covers score tiles 2kk, 2kk + 1.
#pragma unroll
        for (int kk = 0; kk < kPfFlashKeys / 16; ++kk) {
            unsigned ph[4], pl[4];
            split2(sc[2 * kk][0], sc[2 * kk][1], ph[0], pl[0]);
            split2(sc[2 * kk][2], sc[2 * kk][3], ph[1], pl[1]);
            split2(sc[2 * kk + 1][0], sc[2 * kk + 1][1], ph[2], pl[2]);
            split2(sc[2 * kk + 1][2], sc[2 * kk + 1][3], ph[3], pl[3]);
            // ldmatrix.trans rows: thread t gives key kk*16 + (t / 8 % 2) * 8 + t % 8, columns
            // (pair * 2 + t / 16) * 8: matrices 0-1 are b0/b1 of column tile 2*pair, 2-3 of 2*pair + 1.
            const int vkey = kk * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
            for (int pair = 0; pair < ND / 2; ++pair) {
                unsigned b0, b1, b2, b3;
                ldsm_x4_t(vb + (unsigned)((vkey * LDS + (pair * 2 + (lane >> 4)) * 8) * 2), b0, b1, b2, b3);
                mma_16816(o[2 * pair], ph[0], ph[1], ph[2], ph[3], b0, b1);
                mma_16816(o[2 * pair], pl[0], pl[1], pl[2], pl[3], b0, b1);
                mma_16816(o[2 * pair + 1], ph[0], ph[1], ph[2], ph[3], b2, b3);
                mma_16816(o[2 * pair + 1], pl[0], pl[1], pl[2], pl[3], b2, b3);
            }
        }
        __syncthreads();  // the stage is refilled by the next iteration's load
    }
    const int ra = t0 + warp * 16 + qr, rb = ra + 8;
#pragma unroll
    for (int nd = 0; nd < ND; ++nd) {
        const int c = h * HD + nd * 8 + qc;
        if (ra < T) {
            float* dst = a.out + (size_t)ra * a.heads * HD + c;
            dst[0] = __fdiv_rn(o[nd][0], l_a);
            dst[1] = __fdiv_rn(o[nd][1], l_a);
        }
        if (rb < T) {
            float* dst = a.out + (size_t)rb * a.heads * HD + c;
            dst[0] = __fdiv_rn(o[nd][2], l_b);
            dst[1] = __fdiv_rn(o[nd][3], l_b);
        }
    }
}

inline size_t pf_attn_smem(int hd, int gqa)
{
    return sizeof(float) * ((size_t)2 * kPfAttnKeys * (hd + 1) + (size_t)2 * gqa * hd + (size_t)gqa * kPfAttnKeys +
                            3 * (size_t)gqa);
}

}  // namespace muyo
