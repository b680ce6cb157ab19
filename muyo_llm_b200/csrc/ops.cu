// Op-level kernels behind the reference's per-op node contracts (src/LlamaContracts.h), one
// extern "C" entry point each. These back the reference's op checks (src/MatVec.cpp,
// src/RmsNorm.cpp, src/Rope.cpp, ...) and its node-per-op graph; the fused decode path lives in
// decode.cu.
#include <climits>
#include <cstddef>
#include <new>
#include <cmath>
#include <mutex>

#include "common.cuh"
#include "gemv.cuh"

namespace muyo {

constexpr int kThreads = 256;

__device__ __forceinline__ unsigned long long now_ns_ops()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
constexpr int kMaxStagedK = 56 * 1024;  // floats of x staged in shared memory (224 KB)

// ---- GEMV ------------------------------------------------------------------------------------------

struct MatVecDev {
    int ncols, rows, stride_a, stride_b, stride_d;
    long long batch_stride_a, batch_stride_b, batch_stride_d;
    int ne02, ne12, bc2, bc3;
    int k8;  // vector chunks of 8 (F16) or 4 (F32) columns; 0 selects the scalar path
    unsigned flags;
};

__device__ __forceinline__ long long batch_a_index(const MatVecDev& p, int b)
{
    const int i13 = b / p.ne12, i12 = b % p.ne12;
    return (long long)(i13 / p.bc3) * p.ne02 + i12 / p.bc2;
}

__device__ __forceinline__ float fuse_bias(const MatVecDev& p, float v, const float* f0, const float* f1, long long di)
{
    if (p.flags & MUYO_MATVEC_BIAS0)
        v += f0[di];
    if (p.flags & MUYO_MATVEC_BIAS1)
        v += f1[di];
    return v;
}

// Stages x (n floats) in the split layout of gemv.cuh. With a 16-byte-aligned x each thread issues
// all its float4 loads of a pass before its first store, so a pass costs one memory round trip.
__device__ __forceinline__ void stage_x_split(float* xs, const float* x, int n, int k8)
{
    if (k8 > 0 && aligned16(x)) {
        constexpr int V = 4;
        const int Q = 2 * k8;
        const float4* x4 = reinterpret_cast<const float4*>(x);
        float4* xs4 = reinterpret_cast<float4*>(xs);
        for (int q0 = 0; q0 < Q; q0 += V * blockDim.x) {
            float4 v[V];
#pragma unroll
            for (int j = 0; j < V; ++j) {
                const int q = q0 + threadIdx.x + j * blockDim.x;
                if (q < Q)
                    v[j] = __ldg(x4 + q);
            }
#pragma unroll
            for (int j = 0; j < V; ++j) {
                const int q = q0 + threadIdx.x + j * blockDim.x;
                if (q < Q)
                    xs4[xs_slot4(q, k8)] = v[j];
            }
        }
        for (int k = 8 * k8 + threadIdx.x; k < n; k += blockDim.x)
            xs[k] = x[k];
    } else {
        for (int k = threadIdx.x; k < n; k += blockDim.x)
            xs[xs_index(k, k8)] = x[k];
    }
}

// warp_gemv_f16_range with x read from global memory (float4 pairs 2c, 2c + 1 of chunk c; L1-resident
// after the first warp of the SM) instead of the staged copy; the same products in the same order.
template <int ROWS, int U>
__device__ __forceinline__ void warp_gemv_f16_range_xg(const GemvArgs<ROWS, U, 1>& a, int row0, int nvalid,
                                                       const float* __restrict__ x, int c_begin, int c_end, int lane,
                                                       float (&acc)[1][ROWS])
{
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const uint4* rowp[ROWS];
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
        rowp[r] = reinterpret_cast<const uint4*>(a.w[0] + (size_t)(row0 + (r < nvalid ? r : 0)) * a.ldw);
    for (int base = c_begin; base < c_end; base += WARP * U) {
        uint4 wv[ROWS][U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = base + lane + WARP * u;
#pragma unroll
            for (int r = 0; r < ROWS; ++r)
                wv[r][u] = c < c_end ? ld_stream16(rowp[r] + c) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = base + lane + WARP * u;
            if (c < c_end) {
                const float4 xa = __ldg(x4 + 2 * c);
                const float4 xb = __ldg(x4 + 2 * c + 1);
#pragma unroll
                for (int r = 0; r < ROWS; ++r)
                    acc[0][r] = dot_chunk(wv[r][u], xa, xb, acc[0][r]);
            }
        }
    }
}

// One row tile of the F16 GEMV. Row group rg = warp / KSPLIT holds ROWS rows from row0; its KSPLIT
// warps add the contiguous chunk ranges [c_begin, c_end) of those rows, and their sums meet in
// shared memory in a fixed order. On return the group's ks == 0 warp holds the rows' sums in every
// lane. Every warp of the CTA calls it the same number of times (barriers inside when KSPLIT > 1).
template <int ROWS, int U, int KSPLIT, bool XG>
__device__ __forceinline__ void mat_vec_tile_f16(const GemvArgs<ROWS, U, 1>& ga, int row0, int nvalid,
                                                 const float* xs, const float* xg, int k8, int ncols, int c_begin,
                                                 int c_end, int lane, int warp, int ks, float (*ksum)[ROWS],
                                                 float (&acc)[1][ROWS])
{
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
        acc[0][r] = 0.0f;
    if (nvalid > 0) {
        if (XG) {
            warp_gemv_f16_range_xg<ROWS, U>(ga, row0, nvalid, xg, c_begin, c_end, lane, acc);
        } else {
            warp_gemv_f16_range<ROWS, U, 1>(ga, row0, nvalid, xs, k8, c_begin, c_end, lane, acc);
            if (ks == KSPLIT - 1)  // columns past the last full chunk
                warp_gemv_f16_tail<ROWS, 1>(ga.w, ga.ldw, row0, nvalid, xs, k8, ncols, lane, acc);
        }
        warp_reduce_acc<ROWS, 1>(acc);
    }
    if (KSPLIT > 1) {
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < ROWS; ++r)
                ksum[warp][r] = acc[0][r];
        }
        __syncthreads();
        if (ks == 0) {
#pragma unroll
            for (int r = 0; r < ROWS; ++r) {
                float t = ksum[warp][r];
#pragma unroll
                for (int j = 1; j < KSPLIT; ++j)
                    t += ksum[warp + j][r];
                acc[0][r] = t;
            }
        }
        __syncthreads();
    }
}

// XG: x is read from global memory (K a multiple of 8, x 16-byte aligned, one batch, small weights):
// the first weight and x loads leave together, with no staging round trip and no block barrier
// before them.
template <int ROWS, int U, int KSPLIT, bool XG>
__global__ void __launch_bounds__(kThreads) k_mat_vec_f16(MatVecDev p, const __half* __restrict__ A,
                                                          const float* __restrict__ B, float* __restrict__ D,
                                                          const float* __restrict__ f0, const float* __restrict__ f1)
{
    // 8 warps = (8 / KSPLIT) row groups of ROWS rows; the KSPLIT warps of a group split the row's
    // chunks into contiguous ranges, and their sums meet in shared memory in a fixed order.
    constexpr int RG = kThreads / 32 / KSPLIT;
    extern __shared__ float xs[];
    __shared__ float ksum[kThreads / 32][ROWS];
    const int b = blockIdx.y;
    const __half* Ab = A + batch_a_index(p, b) * p.batch_stride_a;
    const float* Bb = B + (long long)b * p.batch_stride_b;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int rg = warp / KSPLIT, ks = warp % KSPLIT;
    const int block_rows = RG * ROWS, ntiles = (p.rows + block_rows - 1) / block_rows;
    // The vector path's rows are 16-byte aligned: start streaming this CTA's first row block into L2
    // while x is staged.
    if (p.k8 > 0 && threadIdx.x == 0 && (int)blockIdx.x < ntiles)
        prefetch_rows_l2(Ab, (size_t)p.stride_a, blockIdx.x * block_rows,
                         min(block_rows, p.rows - (int)blockIdx.x * block_rows));
    pdl_wait();  // the L2 prefetch above is only a hint; every read of A, x or D comes after this wait
    pdl_trigger();
    if (!XG) {
        stage_x_split(xs, Bb, p.ncols, p.k8);
        __syncthreads();
    }
    const int c_begin = (int)((long long)p.k8 * ks / KSPLIT), c_end = (int)((long long)p.k8 * (ks + 1) / KSPLIT);
    GemvArgs<ROWS, U, 1> ga{{Ab}, (size_t)p.stride_a};
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {  // the same trip count in every warp
        const int row0 = tile * block_rows + rg * ROWS;
        const int nvalid = min(ROWS, p.rows - row0);
        const int next0 = (tile + (int)gridDim.x) * block_rows;  // the CTA's next row block
        if (p.k8 > 0 && warp == 0 && lane == 0 && next0 < p.rows)
            prefetch_rows_l2(Ab, (size_t)p.stride_a, next0, min(block_rows, p.rows - next0));
        float acc[1][ROWS];
        mat_vec_tile_f16<ROWS, U, KSPLIT, XG>(ga, row0, nvalid, xs, Bb, p.k8, p.ncols, c_begin, c_end, lane, warp, ks,
                                              ksum, acc);
        if (ks == 0 && lane == 0 && nvalid > 0) {
#pragma unroll
            for (int r = 0; r < ROWS; ++r)
                if (r < nvalid) {
                    const long long di = (long long)b * p.batch_stride_d + row0 + r;
                    D[di] = fuse_bias(p, acc[0][r], f0, f1, di);
                }
        }
    }
}

// F32 weights: lane l takes the 4-column chunks l, l+32, ... (16-byte loads); x staged plainly.
template <int ROWS, int U>
__global__ void __launch_bounds__(kThreads) k_mat_vec_f32(MatVecDev p, const float* __restrict__ A,
                                                          const float* __restrict__ B, float* __restrict__ D,
                                                          const float* __restrict__ f0, const float* __restrict__ f1)
{
    pdl_wait();  // launched with programmatic serialization: wait for the previous kernel
    pdl_trigger();
    extern __shared__ float xs[];
    const int b = blockIdx.y;
    const float* Ab = A + batch_a_index(p, b) * p.batch_stride_a;
    const float* Bb = B + (long long)b * p.batch_stride_b;
    for (int k = threadIdx.x; k < p.ncols; k += blockDim.x)
        xs[k] = Bb[k];
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int K4 = p.k8;
    for (int row0 = (blockIdx.x * nw + warp) * ROWS; row0 < p.rows; row0 += gridDim.x * nw * ROWS) {
        const int nvalid = min(ROWS, p.rows - row0);
        float acc[ROWS];
        const float* rowp[ROWS];
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
            acc[r] = 0.0f;
            rowp[r] = Ab + (size_t)(row0 + (r < nvalid ? r : 0)) * p.stride_a;
        }
        for (int base = 0; base < K4; base += WARP * U) {
            float4 wv[ROWS][U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = base + lane + WARP * u;
#pragma unroll
                for (int r = 0; r < ROWS; ++r)
                    wv[r][u] = c < K4 ? ld_stream16f(rowp[r] + 4 * c) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = base + lane + WARP * u;
                if (c < K4) {
                    const float4 x = reinterpret_cast<const float4*>(xs)[c];
#pragma unroll
                    for (int r = 0; r < ROWS; ++r) {
                        acc[r] = fmaf(wv[r][u].x, x.x, acc[r]);
                        acc[r] = fmaf(wv[r][u].y, x.y, acc[r]);
                        acc[r] = fmaf(wv[r][u].z, x.z, acc[r]);
                        acc[r] = fmaf(wv[r][u].w, x.w, acc[r]);
                    }
                }
            }
        }
        for (int k = 4 * K4 + lane; k < p.ncols; k += WARP) {
#pragma unroll
            for (int r = 0; r < ROWS; ++r)
                acc[r] = fmaf(rowp[r][k], xs[k], acc[r]);
        }
#pragma unroll
        for (int r = 0; r < ROWS; ++r)
            acc[r] = warp_sum(acc[r]);
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < ROWS; ++r)
                if (r < nvalid) {
                    const long long di = (long long)b * p.batch_stride_d + row0 + r;
                    D[di] = fuse_bias(p, acc[r], f0, f1, di);
                }
        }
    }
}

template <typename Kernel>
static cudaError_t set_smem(Kernel k, size_t bytes)
{
    if (bytes <= 48 * 1024)
        return cudaSuccess;
    return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

static int mat_vec_prepare(const MuyoMatVecParams* p, const void* a, const float* b, float* d, const float* f0,
                           const float* f1, size_t esize, MatVecDev& q)
{
    MUYO_REQUIRE(p && a && b && d, "mat_vec: null parameter block or buffer");
    MUYO_REQUIRE(p->ncols > 0 && p->rows > 0, "mat_vec: ncols and rows must be positive");
    if (p->fusion_flags & (MUYO_MATVEC_SCALE0 | MUYO_MATVEC_SCALE1)) {
        set_error("mat_vec: SCALE0/SCALE1 fusion is not implemented");
        return MUYO_EUNSUPPORTED;
    }
    MUYO_REQUIRE((p->fusion_flags & ~0xFu) == 0, "mat_vec: unknown fusion flag bits 0x%x", p->fusion_flags);
    MUYO_REQUIRE(!(p->fusion_flags & MUYO_MATVEC_BIAS0) || f0, "mat_vec: BIAS0 set but fuse0 is null");
    MUYO_REQUIRE(!(p->fusion_flags & MUYO_MATVEC_BIAS1) || f1, "mat_vec: BIAS1 set but fuse1 is null");
    MUYO_REQUIRE(p->ncols <= (uint32_t)kMaxStagedK, "mat_vec: ncols %u exceeds %d", p->ncols, kMaxStagedK);
    q.ncols = (int)p->ncols;
    q.rows = (int)p->rows;
    q.stride_a = (int)(p->stride_a ? p->stride_a : p->ncols);
    q.stride_b = (int)(p->stride_b ? p->stride_b : p->ncols);
    q.stride_d = (int)(p->stride_d ? p->stride_d : p->rows);
    MUYO_REQUIRE((uint32_t)q.stride_a >= p->ncols, "mat_vec: stride_a %d < ncols %u", q.stride_a, p->ncols);
    MUYO_REQUIRE(p->rows <= (uint32_t)q.stride_d, "mat_vec: rows %u exceed stride_d %d", p->rows, q.stride_d);
    q.batch_stride_a = p->batch_stride_a;
    q.batch_stride_b = p->batch_stride_b;
    q.batch_stride_d = p->batch_stride_d;
    q.ne02 = p->ne02 ? (int)p->ne02 : 1;
    q.ne12 = p->ne12 ? (int)p->ne12 : 1;
    q.bc2 = p->broadcast2 ? (int)p->broadcast2 : 1;
    q.bc3 = p->broadcast3 ? (int)p->broadcast3 : 1;
    q.flags = p->fusion_flags;
    const uint32_t batches = p->batches ? p->batches : 1;
    MUYO_REQUIRE(batches <= 65535u, "mat_vec: batches %u exceed 65535", batches);
    MUYO_REQUIRE(batches == 1 || p->batch_stride_d >= p->rows, "mat_vec: batch_stride_d < rows would overlap batches");
    (void)f0;
    (void)f1;
    const int per = esize == 2 ? 8 : 4;  // elements per 16-byte chunk
    const bool vec = aligned16(a) && (q.stride_a % per) == 0 && (q.batch_stride_a % per) == 0;
    q.k8 = vec ? q.ncols / per : 0;
    return MUYO_OK;
}

// Few row blocks per SM (with long rows): 2 or 4 warps per row, so the blocks are smaller and spread
// evenly over the SMs, and more loads are in flight at the start and in the tail. Loads in flight per
// lane then grow with K so that a warp covers a long row in few round trips: U = 8 chunks of 16 bytes
// per row per lane from 8 chunks per lane on, else 4 (each lane still adds its chunks in column order).
static int mat_vec_ksplit(const MatVecDev& q, int batches, int rows_per_warp)
{
    const int tiles1 = (q.rows + 8 * rows_per_warp - 1) / (8 * rows_per_warp);
    return q.k8 < 256 || batches > 1 ? 1 : (tiles1 < 2 * sm_count() ? 4 : (tiles1 < 6 * sm_count() ? 2 : 1));
}

// Rows per warp of the F16 GEMV: 2 once there are two 16-row blocks per SM.
static bool mat_vec_two_rows(const MatVecDev& q) { return (q.rows + 15) / 16 >= 2 * sm_count(); }

template <int ROWS>
static int launch_mat_vec(bool f16, const MatVecDev& q, int batches, const void* a, const float* b, float* d,
                          const float* f0, const float* f1, cudaStream_t s)
{
    const int tiles = (q.rows + 8 * ROWS - 1) / (8 * ROWS);
    int gx = tiles < sm_count() * 8 ? tiles : sm_count() * 8;
    if (batches > 1 && gx * batches > sm_count() * 16)
        gx = (sm_count() * 16 + batches - 1) / batches > 0 ? ((sm_count() * 16 + batches - 1) / batches) : 1;
    if (gx > tiles)
        gx = tiles;
    if (gx < 1)
        gx = 1;
    const size_t smem = (size_t)q.ncols * sizeof(float);
    dim3 grid(gx, batches);
    if (f16) {
        const int ksplit = mat_vec_ksplit(q, batches, ROWS);
        if (ksplit > 1)
            grid.x = (unsigned)((q.rows + 8 / ksplit * ROWS - 1) / (8 / ksplit * ROWS));
        const int lane_chunks = q.k8 / ksplit / 32;
        // Below 16 MB of weights a call is mostly its fixed chain, which reading x from global memory
        // shortens (896x4864: 4.98 -> 4.05 us); for streaming shapes the x reads through L1 cost more
        // than the staging round trip they save (4096x4096: 0.68 -> 0.54 of peak), so x is staged.
        const bool xg = batches == 1 && q.ncols % 8 == 0 && aligned16(b) &&
                        (size_t)q.rows * q.ncols * sizeof(__half) < ((size_t)16 << 20);
        auto k = k_mat_vec_f16<ROWS, 4, 1, false>;
        if (xg) {
            if (ksplit == 4)
                k = lane_chunks >= 8 ? k_mat_vec_f16<ROWS, 8, 4, true> : k_mat_vec_f16<ROWS, 4, 4, true>;
            else if (ksplit == 2)
                k = lane_chunks >= 8 ? k_mat_vec_f16<ROWS, 8, 2, true> : k_mat_vec_f16<ROWS, 4, 2, true>;
            else
                k = lane_chunks >= 8 ? k_mat_vec_f16<ROWS, 8, 1, true> : k_mat_vec_f16<ROWS, 4, 1, true>;
        } else {
            if (ksplit == 4)
                k = lane_chunks >= 8 ? k_mat_vec_f16<ROWS, 8, 4, false> : k_mat_vec_f16<ROWS, 4, 4, false>;
            else if (ksplit == 2)
                k = lane_chunks >= 8 ? k_mat_vec_f16<ROWS, 8, 2, false> : k_mat_vec_f16<ROWS, 4, 2, false>;
            else if (lane_chunks >= 8)
                k = k_mat_vec_f16<ROWS, 8, 1, false>;
        }
        const size_t smem_k = xg ? 0 : smem;
        MUYO_CUDA_TRY(set_smem(k, smem_k));
        // CTAs stride over the row tiles: the grid stops at what is resident at once
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kThreads, smem_k) == cudaSuccess && per_sm > 0 &&
            batches == 1 && grid.x > (unsigned)(per_sm * sm_count()))
            grid.x = per_sm * sm_count();
        MUYO_CUDA_TRY(launch_kernel(k, dim3(grid), dim3(kThreads), smem_k, s, true, q, static_cast<const __half*>(a), b, d, f0, f1));
    } else {
        auto k = k_mat_vec_f32<ROWS, 4>;
        MUYO_CUDA_TRY(set_smem(k, smem));
        MUYO_CUDA_TRY(launch_kernel(k, dim3(grid), dim3(kThreads), smem, s, true, q, static_cast<const float*>(a), b, d, f0, f1));
    }
    MUYO_LAUNCH_CHECK();
    return MUYO_OK;
}

static int mat_vec_any(bool f16, const MuyoMatVecParams* p, const void* a, const float* b, float* d, const float* f0,
                       const float* f1, void* stream)
{
    MatVecDev q{};
    int rc = mat_vec_prepare(p, a, b, d, f0, f1, f16 ? 2 : 4, q);
    if (rc != MUYO_OK)
        return rc;
    const int batches = p->batches ? (int)p->batches : 1;
    const bool two_rows = mat_vec_two_rows(q);
    return two_rows ? launch_mat_vec<2>(f16, q, batches, a, b, d, f0, f1, as_stream(stream))
                    : launch_mat_vec<1>(f16, q, batches, a, b, d, f0, f1, as_stream(stream));
}

// ---- binary head ops -----------------------------------------------------------------------------

struct Dims4 {
    int ne[4];
    long long nb[4];
};

static Dims4 dims(uint32_t n0, uint32_t n1, uint32_t n2, uint32_t n3, uint32_t s0, uint32_t s1, uint32_t s2,
                  uint32_t s3)
{
    Dims4 d;
    d.ne[0] = n0 ? (int)n0 : 1;
    d.ne[1] = n1 ? (int)n1 : 1;
    d.ne[2] = n2 ? (int)n2 : 1;
    d.ne[3] = n3 ? (int)n3 : 1;
    d.nb[0] = s0;
    d.nb[1] = s1;
    d.nb[2] = s2;
    d.nb[3] = s3;
    return d;
}

__global__ void k_add_contig(const float4* __restrict__ a, const float4* __restrict__ b, float4* __restrict__ d,
                             long long n4)
{
    pdl_wait();  // launched with programmatic serialization: wait for the previous kernel
    pdl_trigger();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
        const float4 x = a[i], y = b[i];
        d[i] = make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
    }
}

__global__ void k_add_general(Dims4 A, Dims4 B, Dims4 D, const float* __restrict__ a, const float* __restrict__ b,
                              float* __restrict__ d, long long n)
{
    pdl_wait();  // launched with programmatic serialization: wait for the previous kernel
    pdl_trigger();
    for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < n;
         idx += (long long)gridDim.x * blockDim.x) {
        long long t = idx;
        int i[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            i[k] = (int)(t % D.ne[k]);
            t /= D.ne[k];
        }
        long long ai = 0, bi = 0, di = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            ai += i[k] * A.nb[k];
            bi += (i[k] % B.ne[k]) * B.nb[k];
            di += i[k] * D.nb[k];
        }
        d[di] = a[ai] + b[bi];
    }
}

static bool contiguous(const Dims4& x)
{
    return x.nb[0] == 1 && x.nb[1] == x.ne[0] && x.nb[2] == (long long)x.ne[0] * x.ne[1] &&
           x.nb[3] == (long long)x.ne[0] * x.ne[1] * x.ne[2];
}

static long long count(const Dims4& x) { return (long long)x.ne[0] * x.ne[1] * x.ne[2] * x.ne[3]; }

static int grid_for(long long n, int per_thread = 1)
{
    long long blocks = (n / per_thread + kThreads - 1) / kThreads;
    const long long cap = (long long)sm_count() * 16;
    if (blocks > cap)
        blocks = cap;
    return blocks < 1 ? 1 : (int)blocks;
}

// One CTA per row: sum of squares in F32 (per-thread partials, then a shuffle tree), scale =
// 1/sqrt(mean + eps) in IEEE arithmetic, D = A * scale * W[col % ne10] (rms_norm.comp:87-122,
// src/RmsNorm.cpp:194-205).
__global__ void __launch_bounds__(kThreads) k_rms_norm(Dims4 A, Dims4 W, Dims4 D, const float* __restrict__ a,
                                                       const float* __restrict__ w, float* __restrict__ d, float eps)
{
    pdl_wait();  // launched with programmatic serialization: wait for the previous kernel
    pdl_trigger();
    __shared__ float red[32];
    const int row = blockIdx.x;
    const int i1 = row % A.ne[1], i2 = (row / A.ne[1]) % A.ne[2], i3 = row / (A.ne[1] * A.ne[2]);
    const float* ar = a + i1 * A.nb[1] + i2 * A.nb[2] + i3 * A.nb[3];
    float* dr = d + i1 * D.nb[1] + i2 * D.nb[2] + i3 * D.nb[3];
    const int n = A.ne[0];
    float ss = 0.0f;
    for (int c = threadIdx.x; c < n; c += blockDim.x) {
        const float v = ar[c * A.nb[0]];
        ss = fmaf(v, v, ss);
    }
    ss = block_sum(ss, red);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(ss, (float)n) + eps));
    for (int c = threadIdx.x; c < n; c += blockDim.x)
        dr[c * D.nb[0]] = ar[c * A.nb[0]] * scale * w[(c % W.ne[0]) * W.nb[0]];
}

// Contiguous rows of n4 float4s with a weight of the same length: each thread holds its V float4s of
// the row in registers between the sum of squares and the scaled write, so the row is read from
// memory once. Same arithmetic as k_rms_norm.
template <int V>
__global__ void __launch_bounds__(kThreads) k_rms_norm_rows(const float4* __restrict__ a, const float4* __restrict__ w,
                                                            float4* __restrict__ d, int n4, float eps)
{
    pdl_wait();  // launched with programmatic serialization: wait for the previous kernel
    pdl_trigger();
    __shared__ float red[32];
    const float4* ar = a + (long long)blockIdx.x * n4;
    float4* dr = d + (long long)blockIdx.x * n4;
    float4 v[V];
#pragma unroll
    for (int j = 0; j < V; ++j) {
        const int c = threadIdx.x + j * kThreads;
        v[j] = c < n4 ? ld_stream16f(ar + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < V; ++j) {
        ss = fmaf(v[j].x, v[j].x, ss);
        ss = fmaf(v[j].y, v[j].y, ss);
        ss = fmaf(v[j].z, v[j].z, ss);
        ss = fmaf(v[j].w, v[j].w, ss);
    }
    ss = block_sum(ss, red);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(ss, (float)(4 * n4)) + eps));
#pragma unroll
    for (int j = 0; j < V; ++j) {
        const int c = threadIdx.x + j * kThreads;
        if (c < n4) {
            const float4 g = __ldg(w + c);
            dr[c] = make_float4(v[j].x * scale * g.x, v[j].y * scale * g.y, v[j].z * scale * g.z, v[j].w * scale * g.w);
        }
    }
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v)
{
    return v;
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half v)
{
    return __half2float(v);
}

// get_rows.comp:8-42: D[i10, i11, i12][i00] = A[idx, i11, i12][i00]. An id outside [0, ne01)
// writes zeros (the reference would read out of bounds).
template <typename T>
__global__ void k_get_rows(Dims4 A, Dims4 B, Dims4 D, const T* __restrict__ a, const int32_t* __restrict__ b,
                           float* __restrict__ d)
{
    pdl_wait();  // launched with programmatic serialization: wait for the previous kernel
    pdl_trigger();
    const int i10 = blockIdx.y;
    const int z = blockIdx.z, i11 = z % B.ne[1], i12 = z / B.ne[1];
    const int idx = b[i10 * B.nb[0] + i11 * B.nb[1] + i12 * B.nb[2]];
    const bool ok = idx >= 0 && idx < A.ne[1];
    const T* ar = a + (long long)idx * A.nb[1] + i11 * A.nb[2] + i12 * A.nb[3];
    float* dr = d + i10 * D.nb[1] + i11 * D.nb[2] + i12 * D.nb[3];
    for (int i00 = blockIdx.x * blockDim.x + threadIdx.x; i00 < A.ne[0]; i00 += gridDim.x * blockDim.x)
        dr[i00 * D.nb[0]] = ok ? to_f32(ar[i00 * A.nb[0]]) : 0.0f;
}

// ---- swiglu ----------------------------------------------------------------------------------------

struct GluDev {
    long long N;
    int ne00, ne20, ne21, ne22, mode;
    long long nb0[4], nb1[4], nb2[4];
};

__global__ void k_swiglu(GluDev p, const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ d)
{
    pdl_wait();  // launched with programmatic serialization: wait for the previous kernel
    pdl_trigger();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < p.N; i += (long long)gridDim.x * blockDim.x) {
        const long long per3 = (long long)p.ne22 * p.ne21 * p.ne20, per2 = (long long)p.ne21 * p.ne20;
        const long long i23 = i / per3;
        const long long r3 = i - i23 * per3;
        const long long i22 = r3 / per2;
        const long long r2 = r3 - i22 * per2;
        const long long i21 = r2 / p.ne20;
        const long long i20 = r2 - i21 * p.ne20;
        const long long sa = i23 * p.nb0[3] + i22 * p.nb0[2] + i21 * p.nb0[1] + i20 * p.nb0[0];
        const long long sb = i23 * p.nb1[3] + i22 * p.nb1[2] + i21 * p.nb1[1] + i20 * p.nb1[0];
        const long long sd = i23 * p.nb2[3] + i22 * p.nb2[2] + i21 * p.nb2[1] + i20 * p.nb2[0];
        float g, u;
        if (p.mode == MUYO_GLU_SPLIT) {
            g = a[sa];
            u = b[sb];
        } else {
            const long long off = (long long)(p.ne00 / 2) * p.nb0[0];
            g = p.mode == MUYO_GLU_HALVES ? a[sa] : a[sa + off];
            u = p.mode == MUYO_GLU_HALVES ? a[sa + off] : a[sa];
        }
        d[sd] = silu_mul(g, u);
    }
}

// Split mode with gate, up and output all dense: one flat float4 stream, no index arithmetic.
__global__ void k_swiglu_flat(const float4* __restrict__ a, const float4* __restrict__ b, float4* __restrict__ d,
                              long long n4)
{
    pdl_wait();  // launched with programmatic serialization: wait for the previous kernel
    pdl_trigger();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
        const float4 g = ld_stream16f(a + i), u = ld_stream16f(b + i);
        d[i] = make_float4(silu_mul(g.x, u.x), silu_mul(g.y, u.y), silu_mul(g.z, u.z), silu_mul(g.w, u.w));
    }
}

// ---- RoPE ------------------------------------------------------------------------------------------

struct RopeDev {
    int mode, nrows, n_dims, n_offs, has_ff, is_back;
    float freq_scale, ext_factor, attn_factor, corr0, corr1, theta_scale;
    int ne00, ne01, ne02;
    long long nb01, nb02, nb03, nb11, nb12, nb13, a_offset, d_offset;
};

// rope_funcs.glsl:14-45 (rope_yarn with its ramp), in F32 with accurate cosf/sinf/powf.
__device__ __forceinline__ void rope_yarn(const RopeDev& p, float theta_extrap, int i0, float& c, float& s)
{
    float mscale = p.attn_factor;
    const float theta_interp = p.freq_scale * theta_extrap;
    float theta = theta_interp;
    if (p.ext_factor != 0.0f) {
        const float y = ((float)(i0 / 2) - p.corr0) / fmaxf(0.001f, p.corr1 - p.corr0);
        const float ramp = 1.0f - fminf(1.0f, fmaxf(0.0f, y));
        const float mix = ramp * p.ext_factor;
        theta = theta_interp * (1.0f - mix) + theta_extrap * mix;
        mscale *= 1.0f + 0.1f * logf(1.0f / p.freq_scale);
    }
    if (p.is_back)
        theta = -theta;
    c = cosf(theta) * mscale;
    s = sinf(theta) * mscale;
}

__global__ void k_rope(RopeDev p, const float* __restrict__ x, const int32_t* __restrict__ pos,
                       const float* __restrict__ ff, float* __restrict__ d)
{
    pdl_wait();  // launched with programmatic serialization: wait for the previous kernel
    pdl_trigger();
    const int pairs = p.ne00 / 2;
    const long long total = (long long)p.nrows * pairs;
    for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
         t += (long long)gridDim.x * blockDim.x) {
        const int row = (int)(t / pairs);
        const int i0 = 2 * (int)(t - (long long)row * pairs);
        const int i3 = row / (p.ne01 * p.ne02);
        const int i2 = (row - i3 * p.ne01 * p.ne02) / p.ne01;
        const int i1 = row - i3 * p.ne01 * p.ne02 - i2 * p.ne01;
        const long long xs = p.a_offset + i3 * p.nb03 + i2 * p.nb02 + i1 * p.nb01;
        const long long ds = p.d_offset + i3 * p.nb13 + i2 * p.nb12 + i1 * p.nb11;
        if (i0 < p.n_offs || i0 >= p.n_offs + p.n_dims) {
            d[ds + i0] = x[xs + i0];
            d[ds + i0 + 1] = x[xs + i0 + 1];
            continue;
        }
        const int iw = i0 - p.n_offs;
        const float theta_base = (float)pos[i2] * powf(p.theta_scale, (float)(iw / 2));
        const float freq = p.has_ff ? ff[iw / 2] : 1.0f;
        float c, s;
        rope_yarn(p, theta_base / freq, iw, c, s);
        long long j0, j1;
        if (p.mode == MUYO_ROPE_NEOX) {
            j0 = p.n_offs + iw / 2;
            j1 = j0 + p.n_dims / 2;
        } else {
            j0 = i0;
            j1 = i0 + 1;
        }
        const float x0 = x[xs + j0], x1 = x[xs + j1];
        d[ds + j0] = x0 * c - x1 * s;
        d[ds + j1] = x0 * s + x1 * c;
    }
}

// ---- soft_max --------------------------------------------------------------------------------------

struct SoftMaxDev {
    int KX, KY, ne01, ne02, ne12, ne13;
    long long nb11, nb12, nb13;
    float scale, max_bias, m0, m1;
    int n_head_log2, nrows_x, has_sinks;
};

// One CTA per row (soft_max.comp:58-169): v = x*scale + slope*mask, max (seeded with the sink),
// sum of exp(v - max) (+ exp(sink - max)), D = exp(v - max) * (1 / sum).
__global__ void __launch_bounds__(kThreads) k_soft_max(SoftMaxDev p, const float* __restrict__ x,
                                                       const float* __restrict__ mask,
                                                       const float* __restrict__ sinks, float* __restrict__ d)
{
    pdl_wait();  // launched with programmatic serialization: wait for the previous kernel
    pdl_trigger();
    __shared__ float red[32];
    const int rowx = blockIdx.x;
    const int i03 = rowx / (p.ne01 * p.ne02);
    const int i02 = (rowx - i03 * p.ne01 * p.ne02) / p.ne01;
    const int i01 = rowx % p.ne01;
    long long rowy = 0;
    if (p.KY > 0)
        rowy = i01 * p.nb11 + (i02 % p.ne12) * p.nb12 + (i03 % p.ne13) * p.nb13;
    float slope = 1.0f;
    if (p.max_bias > 0.0f) {
        const int h = (rowx / p.ne01) % p.ne02;
        const float base = h < p.n_head_log2 ? p.m0 : p.m1;
        const int e = h < p.n_head_log2 ? h + 1 : 2 * (h - p.n_head_log2) + 1;
        slope = powf(base, (float)e);
    }
    const float* xr = x + (long long)rowx * p.KX;
    float* dr = d + (long long)rowx * p.KX;
    float m = p.has_sinks ? sinks[i02] : -INFINITY;
    for (int c = threadIdx.x; c < p.KX; c += blockDim.x) {
        const float v = xr[c] * p.scale + (p.KY > 0 ? slope * mask[rowy + c] : 0.0f);
        dr[c] = v;
        m = fmaxf(m, v);
    }
    m = block_max(m, red);
    float sum = 0.0f;
    for (int c = threadIdx.x; c < p.KX; c += blockDim.x) {
        const float e = expf(dr[c] - m);
        dr[c] = e;
        sum += e;
    }
    sum = block_sum(sum, red);
    if (p.has_sinks)
        sum += expf(sinks[i02] - m);
    const float rcp = __fdiv_rn(1.0f, sum);
    for (int c = threadIdx.x; c < p.KX; c += blockDim.x)
        dr[c] = dr[c] * rcp;
}

// ---- argmax ----------------------------------------------------------------------------------------

constexpr int kArgmaxChunk = 8192;  // logits per CTA
struct ArgPair {
    float v;
    int i;
};

// Stage 1: each CTA scans kArgmaxChunk logits of a row (increasing index per thread, strict >),
// then reduces with the first-index tie rule. Stage 2 reduces a row's CTA pairs the same way.
__device__ __forceinline__ ArgPair block_argmax(float v, int i)
{
    __shared__ float sv[32];
    __shared__ int si[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    warp_argmax(v, i);
    __syncthreads();
    if (lane == 0) {
        sv[warp] = v;
        si[warp] = i;
    }
    __syncthreads();
    v = lane < nw ? sv[lane] : -INFINITY;
    i = lane < nw ? si[lane] : INT_MAX;
    warp_argmax(v, i);
    return ArgPair{v, i};
}

__global__ void __launch_bounds__(kThreads) k_argmax_partial(const float* __restrict__ a, int KX, int per_row,
                                                             int index_base, ArgPair* __restrict__ part)
{
    pdl_wait();  // launched with programmatic serialization: wait for the previous kernel
    pdl_trigger();
    const int row = blockIdx.y, blk = blockIdx.x;
    const float* ar = a + (long long)row * KX;
    const int c0 = blk * kArgmaxChunk, c1 = min(KX, c0 + kArgmaxChunk);
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int c = c0 + threadIdx.x; c < c1; c += blockDim.x) {
        const float v = ar[c];
        if (pair_better(v, c, bv, bi))
            bv = v, bi = c;
    }
    ArgPair r = block_argmax(bv, bi);
    if (threadIdx.x == 0) {
        if (r.i != INT_MAX)
            r.i += index_base;
        part[(long long)row * per_row + blk] = r;
    }
}

// Stage 1 for rows whose length is a multiple of 4 and whose base is 16-byte aligned: the CTA's
// kArgmaxChunk logits as float4 loads, all of a thread's loads issued before its compares.
constexpr int kArgmaxVec = kArgmaxChunk / 4 / kThreads;  // float4s per thread
__global__ void __launch_bounds__(kThreads) k_argmax_partial4(const float* __restrict__ a, int KX, int per_row,
                                                              int index_base, ArgPair* __restrict__ part)
{
    pdl_wait();  // launched with programmatic serialization: wait for the previous kernel
    pdl_trigger();
    const int row = blockIdx.y, blk = blockIdx.x;
    const float4* ar = reinterpret_cast<const float4*>(a + (long long)row * KX);
    const int q0 = blk * (kArgmaxChunk / 4), q1 = min(KX / 4, q0 + kArgmaxChunk / 4);
    float4 v[kArgmaxVec];
#pragma unroll
    for (int j = 0; j < kArgmaxVec; ++j) {
        const int q = q0 + threadIdx.x + j * kThreads;
        v[j] = q < q1 ? ld_stream16f(ar + q) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    }
    float bv = -INFINITY;
    int bi = INT_MAX;
#pragma unroll
    for (int j = 0; j < kArgmaxVec; ++j) {
        const int q = q0 + threadIdx.x + j * kThreads;
        if (q < q1) {
            const float e[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
            for (int t = 0; t < 4; ++t)
                if (pair_better(e[t], 4 * q + t, bv, bi))
                    bv = e[t], bi = 4 * q + t;
        }
    }
    ArgPair r = block_argmax(bv, bi);
    if (threadIdx.x == 0) {
        if (r.i != INT_MAX)
            r.i += index_base;
        part[(long long)row * per_row + blk] = r;
    }
}

// Reduces n pairs per row; writes the index (0 when no value compares, e.g. all NaN, as the
// host's scan that starts from index 0 would return).
__global__ void __launch_bounds__(kThreads) k_argmax_final(const ArgPair* __restrict__ part, int n,
                                                           int32_t* __restrict__ d)
{
    pdl_wait();  // launched with programmatic serialization: wait for the previous kernel
    pdl_trigger();
    const int row = blockIdx.x;
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int k = threadIdx.x; k < n; k += blockDim.x) {
        const ArgPair q = part[(long long)row * n + k];
        if (pair_better(q.v, q.i, bv, bi))
            bv = q.v, bi = q.i;
    }
    ArgPair r = block_argmax(bv, bi);
    if (threadIdx.x == 0)
        d[row] = r.i == INT_MAX ? 0 : r.i;
}

// ---- copy ------------------------------------------------------------------------------------------

__global__ void k_copy(Dims4 S, Dims4 T, long long a_off, long long d_off, const float* __restrict__ a,
                       float* __restrict__ d, long long n)
{
    pdl_wait();  // launched with programmatic serialization: wait for the previous kernel
    pdl_trigger();
    for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < n;
         idx += (long long)gridDim.x * blockDim.x) {
        long long t = idx, u = idx, si = a_off, di = d_off;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            si += (t % S.ne[k]) * S.nb[k];
            t /= S.ne[k];
            di += (u % T.ne[k]) * T.nb[k];
            u /= T.ne[k];
        }
        d[di] = a[si];
    }
}

// Reduces n partial pairs into one pair (the shard result of mat_vec_f16_argmax).
__global__ void __launch_bounds__(kThreads) k_pairs_to_pair(const ArgPair* __restrict__ part, int n, ArgPair* __restrict__ out)
{
    pdl_wait();  // launched with programmatic serialization: wait for the previous kernel
    pdl_trigger();
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int k = threadIdx.x; k < n; k += blockDim.x) {
        const ArgPair q = part[k];
        if (pair_better(q.v, q.i, bv, bi))
            bv = q.v, bi = q.i;
    }
    const ArgPair r = block_argmax(bv, bi);
    if (threadIdx.x == 0)
        *out = r;
}


// ---- row-sharded GEMV fused with its all-gather over NVLink peer memory ---------------------------
// One GPU's share of y = W x over `world` GPUs of one node (one process each). Every rank owns a
// P2PBuffer (header + two [rows_total] output slots), and every rank's buffer is mapped into every
// other rank through CUDA IPC. Call number `epoch` (the rank's own count of calls, kept in its header
// on the device, so that calls captured in a CUDA graph count too) uses output slot and pair slot
// epoch & 1: a peer can be at most one call ahead (it cannot finish call e + 1 before this rank
// publishes e + 1, which this rank does only after its own call e and whatever the caller queued
// after it), so a peer's next call writes the other slot while this rank still reads call e's. A call
// is one kernel per GPU:
//   1. each CTA computes its rows and stores every value into every rank's output (NVLink stores);
//   2. each CTA leaves its best (value, global index) in the local header, fences at system scope
//      and counts itself in;
//   3. the last CTA fences at system scope (every CTA's rows now precede what it stores next),
//      reduces the rank's pair and stores it into every rank's pair slot as two 64-bit words
//      {epoch, value bits} and {epoch, index}: each word is single-copy atomic, so a reader that
//      sees the epoch in both sees the pair, and the pair doubles as the rank's "rows are in" flag;
//   4. it then waits (bounded) until every rank's words in its own header carry the epoch, fences
//      at system scope (the peers' rows become visible to what follows), and writes the first-index
//      maximum over the ranks' pairs as the token.
// The epoch counts the calls, identically on every rank, so the slots never need resetting.
constexpr int kP2PMaxRanks = 8;
constexpr unsigned long long kP2PWaitNs = 2000000000ull;

struct alignas(16) P2PHeader {
    // pair[e & 1][r]: rank r's pair of call e as {e << 32 | value bits, e << 32 | index}
    unsigned long long pair[2][kP2PMaxRanks][2];
    int counter;      // arrivals of this rank's CTAs (reset by the last one)
    int err;          // 5: a wait for a peer's pair expired
    unsigned calls;   // this rank's calls so far (written by the last CTA of each call)
    int pad[29];
};

struct P2PArgs {
    const __half* A;  // local shard [local_rows][lda]
    const float* x;
    int K, k8, local_rows, row_begin, rows_total, world, rank;
    long long lda;
    long long slot_floats;           // floats from output slot 0 to slot 1
    float* y[kP2PMaxRanks];          // every rank's output slot 0 (this rank's slice goes to each)
    P2PHeader* hdr[kP2PMaxRanks];    // every rank's header
    ArgPair* cta_pairs;              // local scratch: one pair per CTA
    int32_t* token;
};

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v)
{
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ void ld_relaxed_sys_v2u64(const unsigned long long* p, unsigned long long& a,
                                                     unsigned long long& b)
{
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Rows of a CTA's output gathered in shared memory before they leave for every rank (a multiple of
// every tile height 8 / KSPLIT * ROWS).
constexpr int kP2PChunkRows = 256;

// Step 1 runs the row tiles of k_mat_vec_f16 with the same ROWS, U and KSPLIT (mat_vec_ksplit), so a
// shard's values are bit-identical to muyo_cuda_mat_vec_f16 on that shard. Each CTA takes a
// contiguous range of tiles; its values collect in shared memory and leave in runs of up to
// kP2PChunkRows rows, consecutive threads storing consecutive rows of one rank's slot.
template <int ROWS, int U, int KSPLIT>
__global__ void __launch_bounds__(kThreads) k_gemv_allgather(P2PArgs p)
{
    constexpr int RG = kThreads / 32 / KSPLIT, BR = RG * ROWS;
    static_assert(kP2PChunkRows % BR == 0, "the chunk holds whole tiles");
    extern __shared__ float xs[];
    __shared__ float ksum[kThreads / 32][ROWS];
    __shared__ float ybuf[kP2PChunkRows];
    __shared__ int last_sm;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int rg = warp / KSPLIT, ks = warp % KSPLIT;
    const int ntiles = (p.local_rows + BR - 1) / BR;
    const int t_begin = (int)((long long)ntiles * blockIdx.x / gridDim.x);
    const int t_end = (int)((long long)ntiles * (blockIdx.x + 1) / gridDim.x);
    if (threadIdx.x == 0 && t_begin < t_end)
        prefetch_rows_l2(p.A, (size_t)p.lda, t_begin * BR, min(BR, p.local_rows - t_begin * BR));
    pdl_wait();  // the L2 prefetch above is only a hint; every read of A, x or the buffers comes after this wait
    pdl_trigger();
    // This call's number: the previous call's last CTA stored its own (stream order makes it visible);
    // this call's last CTA stores the next one only after every CTA of this call has arrived.
    const unsigned epoch = __ldcg(&p.hdr[p.rank]->calls) + 1u;
    const long long slot = (long long)(epoch & 1u) * p.slot_floats;
    stage_x_split(xs, p.x, p.K, p.k8);
    __syncthreads();
    const int c_begin = (int)((long long)p.k8 * ks / KSPLIT), c_end = (int)((long long)p.k8 * (ks + 1) / KSPLIT);
    GemvArgs<ROWS, U, 1> ga{{p.A}, (size_t)p.lda};
    float bv = -INFINITY;
    int bi = INT_MAX;
    int chunk0 = t_begin * BR;  // first local row held in ybuf
    for (int tile = t_begin; tile < t_end; ++tile) {  // the same trip count in every warp
        const int row0 = tile * BR + rg * ROWS;
        const int nvalid = min(ROWS, p.local_rows - row0);
        const int next0 = (tile + 1) * BR;
        if (warp == 0 && lane == 0 && tile + 1 < t_end)
            prefetch_rows_l2(p.A, (size_t)p.lda, next0, min(BR, p.local_rows - next0));
        float acc[1][ROWS];
        mat_vec_tile_f16<ROWS, U, KSPLIT, false>(ga, row0, nvalid, xs, p.x, p.k8, p.K, c_begin, c_end, lane, warp, ks,
                                                 ksum, acc);
        if (ks == 0 && lane == 0) {
#pragma unroll
            for (int r = 0; r < ROWS; ++r)
                if (r < nvalid) {
                    ybuf[row0 + r - chunk0] = acc[0][r];
                    if (pair_better(acc[0][r], p.row_begin + row0 + r, bv, bi))
                        bv = acc[0][r], bi = p.row_begin + row0 + r;
                }
        }
        const int held = next0 - chunk0;
        if (held == kP2PChunkRows || tile + 1 == t_end) {  // uniform across the CTA
            __syncthreads();
            const int n = min(held, p.local_rows - chunk0);
            for (int t = threadIdx.x; t < p.world * n; t += blockDim.x) {
                const int r = t / n, i = t - r * n;
                p.y[r][slot + p.row_begin + chunk0 + i] = ybuf[i];
            }
            __syncthreads();
            chunk0 = next0;
        }
    }
    const ArgPair cta = block_argmax(bv, bi);  // uniform across the CTA after its last __syncthreads
    __syncthreads();
    if (threadIdx.x == 0) {
        p.cta_pairs[blockIdx.x] = cta;
        __threadfence_system();  // this CTA's output stores (to every rank) before its arrival
        last_sm = atomicAdd(&p.hdr[p.rank]->counter, 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (!last_sm)
        return;
    __threadfence_system();
    float v = -INFINITY;
    int i = INT_MAX;
    for (int k = threadIdx.x; k < (int)gridDim.x; k += blockDim.x) {
        const ArgPair q{__ldcg(&p.cta_pairs[k].v), __ldcg(&p.cta_pairs[k].i)};
        if (pair_better(q.v, q.i, v, i))
            v = q.v, i = q.i;
    }
    const ArgPair mine = block_argmax(v, i);
    if (threadIdx.x != 0)
        return;
    P2PHeader* own = p.hdr[p.rank];
    own->counter = 0;
    const int ps = epoch & 1u;
    const unsigned long long tag = (unsigned long long)epoch << 32;
    for (int r = 0; r < p.world; ++r) {
        st_relaxed_sys_u64(&p.hdr[r]->pair[ps][p.rank][0], tag | __float_as_uint(mine.v));
        st_relaxed_sys_u64(&p.hdr[r]->pair[ps][p.rank][1], tag | (unsigned)mine.i);
    }
    // Every rank's slice and pair are in this buffer once its pair words carry this epoch (a peer one
    // call ahead writes the other slot).
    const unsigned long long t0 = now_ns_ops();
    bool ok = true;
    float bv2 = -INFINITY;
    int bi2 = INT_MAX;
    for (int r = 0; r < p.world && ok; ++r) {
        unsigned long long wv, wi;
        for (;;) {
            ld_relaxed_sys_v2u64(&own->pair[ps][r][0], wv, wi);
            if ((unsigned)(wv >> 32) == epoch && (unsigned)(wi >> 32) == epoch)
                break;
            if (now_ns_ops() - t0 > kP2PWaitNs) {
                ok = false;
                atomicMax(&own->err, 5);
                break;
            }
        }
        if (ok && pair_better(__uint_as_float((unsigned)wv), (int)(unsigned)wi, bv2, bi2))
            bv2 = __uint_as_float((unsigned)wv), bi2 = (int)(unsigned)wi;
    }
    __threadfence_system();  // the peers' rows, published before their pair words, precede what follows
    if (!ok)
        bi2 = INT_MAX;
    *p.token = bi2 == INT_MAX ? 0 : bi2;
    own->calls = epoch;
}
}  // namespace muyo

using namespace muyo;

// ---- extern "C" entry points ---------------------------------------------------------------------

extern "C" int muyo_cuda_mat_vec_f16(const MuyoMatVecParams* p, const void* a, const float* b, float* d,
                                     const float* fuse0, const float* fuse1, void* stream)
{
    clear_error();
    return mat_vec_any(true, p, a, b, d, fuse0, fuse1, stream);
}

extern "C" int muyo_cuda_mat_vec_f32(const MuyoMatVecParams* p, const float* a, const float* b, float* d,
                                     const float* fuse0, const float* fuse1, void* stream)
{
    clear_error();
    return mat_vec_any(false, p, a, b, d, fuse0, fuse1, stream);
}

extern "C" int muyo_cuda_add(const MuyoBinaryParams* p, const float* a, const float* b, float* d, void* stream)
{
    clear_error();
    MUYO_REQUIRE(p && a && b && d, "add: null parameter block or buffer");
    const Dims4 A = dims(p->ne00, p->ne01, p->ne02, p->ne03, p->nb00, p->nb01, p->nb02, p->nb03);
    const Dims4 B = dims(p->ne10, p->ne11, p->ne12, p->ne13, p->nb10, p->nb11, p->nb12, p->nb13);
    const Dims4 D = dims(p->ne20, p->ne21, p->ne22, p->ne23, p->nb20, p->nb21, p->nb22, p->nb23);
    const long long n = count(D);
    MUYO_REQUIRE(n > 0, "add: empty output");
    MUYO_REQUIRE(count(A) == n, "add: A and D element counts differ");
    for (int k = 0; k < 4; ++k)
        MUYO_REQUIRE(A.ne[k] == D.ne[k] && D.ne[k] % B.ne[k] == 0, "add: dimension %d does not broadcast", k);
    const cudaStream_t s = as_stream(stream);
    if (contiguous(A) && contiguous(B) && contiguous(D) && count(B) == n && n % 4 == 0 && aligned16(a) &&
        aligned16(b) && aligned16(d)) {
        MUYO_CUDA_TRY(launch_kernel(k_add_contig, dim3(grid_for(n / 4)), dim3(kThreads), 0, s, true, reinterpret_cast<const float4*>(a),
                                                          reinterpret_cast<const float4*>(b),
                                                          reinterpret_cast<float4*>(d), n / 4));
    } else {
        MUYO_CUDA_TRY(launch_kernel(k_add_general, dim3(grid_for(n)), dim3(kThreads), 0, s, true, A, B, D, a, b, d, n));
    }
    MUYO_LAUNCH_CHECK();
    return MUYO_OK;
}

extern "C" int muyo_cuda_rms_norm(const MuyoBinaryParams* p, const float* a, const float* w, float* d, void* stream)
{
    clear_error();
    MUYO_REQUIRE(p && a && w && d, "rms_norm: null parameter block or buffer");
    const Dims4 A = dims(p->ne00, p->ne01, p->ne02, p->ne03, p->nb00 ? p->nb00 : 1, p->nb01, p->nb02, p->nb03);
    const Dims4 W = dims(p->ne10, 1, 1, 1, p->nb10 ? p->nb10 : 1, 0, 0, 0);
    const Dims4 D = dims(p->ne20, p->ne21, p->ne22, p->ne23, p->nb20 ? p->nb20 : 1, p->nb21, p->nb22, p->nb23);
    MUYO_REQUIRE(p->ne00 > 0 && p->ne10 > 0, "rms_norm: empty row or weight");
    MUYO_REQUIRE(D.ne[0] == A.ne[0] && D.ne[1] == A.ne[1] && D.ne[2] == A.ne[2] && D.ne[3] == A.ne[3],
                 "rms_norm: D shape differs from A");
    MUYO_REQUIRE(p->param1 >= 0.0f, "rms_norm: eps must be >= 0");
    const long long rows = (long long)A.ne[1] * A.ne[2] * A.ne[3];
    MUYO_REQUIRE(rows <= INT_MAX, "rms_norm: too many rows");
    const int n = A.ne[0], n4 = n / 4;
    const cudaStream_t s = as_stream(stream);
    if (contiguous(A) && contiguous(D) && W.ne[0] == n && W.nb[0] == 1 && n % 4 == 0 && n4 <= 8 * kThreads &&
        aligned16(a) && aligned16(w) && aligned16(d)) {
        const float4 *a4 = reinterpret_cast<const float4*>(a), *w4 = reinterpret_cast<const float4*>(w);
        float4* d4 = reinterpret_cast<float4*>(d);
        if (n4 <= kThreads)
            MUYO_CUDA_TRY(launch_kernel(k_rms_norm_rows<1>, dim3((unsigned)rows), dim3(kThreads), 0, s, true, a4, w4, d4, n4, p->param1));
        else if (n4 <= 2 * kThreads)
            MUYO_CUDA_TRY(launch_kernel(k_rms_norm_rows<2>, dim3((unsigned)rows), dim3(kThreads), 0, s, true, a4, w4, d4, n4, p->param1));
        else if (n4 <= 4 * kThreads)
            MUYO_CUDA_TRY(launch_kernel(k_rms_norm_rows<4>, dim3((unsigned)rows), dim3(kThreads), 0, s, true, a4, w4, d4, n4, p->param1));
        else
            MUYO_CUDA_TRY(launch_kernel(k_rms_norm_rows<8>, dim3((unsigned)rows), dim3(kThreads), 0, s, true, a4, w4, d4, n4, p->param1));
    } else {
        MUYO_CUDA_TRY(launch_kernel(k_rms_norm, dim3((unsigned)rows), dim3(kThreads), 0, s, true, A, W, D, a, w, d, p->param1));
    }
    MUYO_LAUNCH_CHECK();
    return MUYO_OK;
}

static int get_rows_any(bool f16, const MuyoBinaryParams* p, const void* a, const int32_t* b, float* d, void* stream)
{
    MUYO_REQUIRE(p && a && b && d, "get_rows: null parameter block or buffer");
    const Dims4 A = dims(p->ne00, p->ne01, p->ne02, p->ne03, p->nb00 ? p->nb00 : 1, p->nb01, p->nb02, p->nb03);
    const Dims4 B = dims(p->ne10, p->ne11, p->ne12, p->ne13, p->nb10 ? p->nb10 : 1, p->nb11, p->nb12, p->nb13);
    const Dims4 D = dims(p->ne20, p->ne21, p->ne22, p->ne23, p->nb20 ? p->nb20 : 1, p->nb21, p->nb22, p->nb23);
    MUYO_REQUIRE(p->ne00 > 0 && p->ne01 > 0, "get_rows: empty table");
    MUYO_REQUIRE(D.ne[0] == A.ne[0], "get_rows: output row length %d != table row length %d", D.ne[0], A.ne[0]);
    MUYO_REQUIRE(B.ne[0] <= 65535 && (long long)B.ne[1] * B.ne[2] <= 65535, "get_rows: too many ids");
    dim3 grid((A.ne[0] + kThreads - 1) / kThreads, B.ne[0], B.ne[1] * B.ne[2]);
    if (f16)
        MUYO_CUDA_TRY(launch_kernel(k_get_rows<__half>, dim3(grid), dim3(kThreads), 0, as_stream(stream), true, A, B, D, static_cast<const __half*>(a), b, d));
    else
        MUYO_CUDA_TRY(launch_kernel(k_get_rows<float>, dim3(grid), dim3(kThreads), 0, as_stream(stream), true, A, B, D, static_cast<const float*>(a), b, d));
    MUYO_LAUNCH_CHECK();
    return MUYO_OK;
}

extern "C" int muyo_cuda_get_rows_f16(const MuyoBinaryParams* p, const void* a, const int32_t* b, float* d,
                                      void* stream)
{
    clear_error();
    return get_rows_any(true, p, a, b, d, stream);
}

extern "C" int muyo_cuda_get_rows_f32(const MuyoBinaryParams* p, const float* a, const int32_t* b, float* d,
                                      void* stream)
{
    clear_error();
    return get_rows_any(false, p, a, b, d, stream);
}

extern "C" int muyo_cuda_swiglu(const MuyoGluParams* p, const float* a, const float* b, float* d, void* stream)
{
    clear_error();
    MUYO_REQUIRE(p && a && d, "swiglu: null parameter block or buffer");
    MUYO_REQUIRE(p->mode <= MUYO_GLU_SPLIT, "swiglu: unknown mode %u", p->mode);
    MUYO_REQUIRE(p->mode != MUYO_GLU_SPLIT || b, "swiglu: split mode needs B");
    MUYO_REQUIRE(p->N > 0 && p->ne20 > 0, "swiglu: empty output");
    MUYO_REQUIRE(p->mode == MUYO_GLU_SPLIT || p->ne00 >= 2 * p->ne20, "swiglu: A row too short for [gate|up]");
    GluDev g{};
    g.N = p->N;
    g.ne00 = (int)p->ne00;
    g.ne20 = (int)p->ne20;
    g.ne21 = p->ne21 ? (int)p->ne21 : 1;
    g.ne22 = p->ne22 ? (int)p->ne22 : 1;
    g.mode = (int)p->mode;
    const uint32_t nb0[4] = {p->nb00, p->nb01, p->nb02, p->nb03}, nb1[4] = {p->nb10, p->nb11, p->nb12, p->nb13},
                   nb2[4] = {p->nb20, p->nb21, p->nb22, p->nb23};
    for (int k = 0; k < 4; ++k) {
        g.nb0[k] = nb0[k];
        g.nb1[k] = nb1[k];
        g.nb2[k] = nb2[k];
    }
    if (!g.nb0[0])
        g.nb0[0] = 1;
    if (!g.nb1[0])
        g.nb1[0] = 1;
    if (!g.nb2[0])
        g.nb2[0] = 1;
    // Flat when element i of D, A and B sits at offset i of each: unit element stride, and each row
    // level that the N elements reach is packed right after the level below it.
    const long long rows_n = (g.N + g.ne20 - 1) / g.ne20;
    auto dense = [&](const long long* nb) {
        return nb[0] == 1 && (g.ne21 == 1 || nb[1] == g.ne20) &&
               (g.ne22 == 1 || nb[2] == (long long)g.ne20 * g.ne21) &&
               (rows_n <= (long long)g.ne21 * g.ne22 || nb[3] == (long long)g.ne20 * g.ne21 * g.ne22);
    };
    const cudaStream_t s = as_stream(stream);
    if (g.mode == MUYO_GLU_SPLIT && g.N % 4 == 0 && dense(g.nb0) && dense(g.nb1) && dense(g.nb2) && aligned16(a) &&
        aligned16(b) && aligned16(d)) {
        MUYO_CUDA_TRY(launch_kernel(k_swiglu_flat, dim3(grid_for(g.N / 4)), dim3(kThreads), 0, s, true, reinterpret_cast<const float4*>(a),
                                                             reinterpret_cast<const float4*>(b),
                                                             reinterpret_cast<float4*>(d), g.N / 4));
    } else {
        MUYO_CUDA_TRY(launch_kernel(k_swiglu, dim3(grid_for(g.N)), dim3(kThreads), 0, s, true, g, a, b, d));
    }
    MUYO_LAUNCH_CHECK();
    return MUYO_OK;
}

extern "C" int muyo_cuda_rope(const MuyoRopeParams* p, const float* x, const int32_t* pos, const float* freq_factors,
                              float* d, void* stream)
{
    clear_error();
    MUYO_REQUIRE(p && x && pos && d, "rope: null parameter block or buffer");
    MUYO_REQUIRE(p->rope_mode == MUYO_ROPE_NEOX || p->rope_mode == MUYO_ROPE_NORMAL,
                 "rope: mode %u not implemented (NORMAL=0, NEOX=2)", p->rope_mode);
    MUYO_REQUIRE(p->ne00 > 0 && p->ne00 % 2 == 0, "rope: ne00 must be positive and even");
    MUYO_REQUIRE(p->n_dims % 2 == 0 && p->n_offs % 2 == 0 && p->n_offs + p->n_dims <= p->ne00,
                 "rope: rotated channels [n_offs, n_offs + n_dims) must be even and within ne00");
    MUYO_REQUIRE(!p->has_ff || freq_factors, "rope: has_ff set but freq_factors is null");
    MUYO_REQUIRE(p->nrows > 0, "rope: no rows");
    RopeDev r{};
    r.mode = (int)p->rope_mode;
    r.nrows = (int)p->nrows;
    r.n_dims = (int)p->n_dims;
    r.n_offs = (int)p->n_offs;
    r.has_ff = (int)p->has_ff;
    r.is_back = (int)p->is_back;
    r.freq_scale = p->freq_scale;
    r.ext_factor = p->ext_factor;
    r.attn_factor = p->attn_factor;
    r.corr0 = p->corr_dims[0];
    r.corr1 = p->corr_dims[1];
    r.theta_scale = p->theta_scale;
    r.ne00 = (int)p->ne00;
    r.ne01 = p->ne01 ? (int)p->ne01 : 1;
    r.ne02 = p->ne02 ? (int)p->ne02 : 1;
    r.nb01 = p->nb01;
    r.nb02 = p->nb02;
    r.nb03 = p->nb03;
    r.nb11 = p->nb11;
    r.nb12 = p->nb12;
    r.nb13 = p->nb13;
    r.a_offset = p->a_offset;
    r.d_offset = p->d_offset;
    const long long total = (long long)p->nrows * (p->ne00 / 2);
    MUYO_CUDA_TRY(launch_kernel(k_rope, dim3(grid_for(total)), dim3(kThreads), 0, as_stream(stream), true, r, x, pos, freq_factors, d));
    MUYO_LAUNCH_CHECK();
    return MUYO_OK;
}

extern "C" int muyo_cuda_soft_max(const MuyoSoftMaxParams* p, const float* x, const float* mask, const float* sinks,
                                  float* d, void* stream)
{
    clear_error();
    MUYO_REQUIRE(p && x && d, "soft_max: null parameter block or buffer");
    MUYO_REQUIRE(p->KX > 0 && p->nrows_x > 0, "soft_max: empty rows");
    MUYO_REQUIRE(p->KY == 0 || mask, "soft_max: KY > 0 needs a mask");
    MUYO_REQUIRE(!p->has_sinks || sinks, "soft_max: has_sinks needs sinks");
    MUYO_REQUIRE(x != d, "soft_max: in-place (x == d) is not supported");
    SoftMaxDev s{};
    s.KX = (int)p->KX;
    s.KY = (int)p->KY;
    s.ne01 = p->ne01 ? (int)p->ne01 : 1;
    s.ne02 = p->ne02 ? (int)p->ne02 : 1;
    s.ne12 = p->ne12 ? (int)p->ne12 : 1;
    s.ne13 = p->ne13 ? (int)p->ne13 : 1;
    s.nb11 = p->nb11;
    s.nb12 = p->nb12;
    s.nb13 = p->nb13;
    s.scale = p->scale;
    s.max_bias = p->max_bias;
    s.m0 = p->m0;
    s.m1 = p->m1;
    s.n_head_log2 = (int)p->n_head_log2;
    s.nrows_x = (int)p->nrows_x;
    s.has_sinks = (int)p->has_sinks;
    MUYO_CUDA_TRY(launch_kernel(k_soft_max, dim3(p->nrows_x), dim3(kThreads), 0, as_stream(stream), true, s, x, mask, sinks, d));
    MUYO_LAUNCH_CHECK();
    return MUYO_OK;
}

static int argmax_blocks(uint32_t KX) { return (int)((KX + kArgmaxChunk - 1) / kArgmaxChunk); }

extern "C" size_t muyo_cuda_argmax_workspace_size(const MuyoGenericParams* p)
{
    if (!p || p->KX == 0)
        return 0;
    const size_t ky = p->KY ? p->KY : 1;
    return ky * (size_t)argmax_blocks(p->KX) * sizeof(ArgPair);
}

static int argmax_launch(const float* a, uint32_t KX, uint32_t KY, int index_base, ArgPair* part, int32_t* d,
                         cudaStream_t s)
{
    const int per_row = argmax_blocks(KX);
    if (KX % 4 == 0 && aligned16(a))
        MUYO_CUDA_TRY(launch_kernel(k_argmax_partial4, dim3(dim3(per_row, KY)), dim3(kThreads), 0, s, true, a, (int)KX, per_row, index_base, part));
    else
        MUYO_CUDA_TRY(launch_kernel(k_argmax_partial, dim3(dim3(per_row, KY)), dim3(kThreads), 0, s, true, a, (int)KX, per_row, index_base, part));
    MUYO_LAUNCH_CHECK();
    if (d) {
        MUYO_CUDA_TRY(launch_kernel(k_argmax_final, dim3(KY), dim3(kThreads), 0, s, true, part, per_row, d));
        MUYO_LAUNCH_CHECK();
    }
    return MUYO_OK;
}

extern "C" int muyo_cuda_argmax(const MuyoGenericParams* p, const float* a, int32_t* d, void* workspace,
                                size_t workspace_bytes, void* stream)
{
    clear_error();
    MUYO_REQUIRE(p && a && d, "argmax: null parameter block or buffer");
    MUYO_REQUIRE(p->KX > 0 && p->KX <= (uint32_t)INT_MAX, "argmax: KX must be in [1, INT_MAX]");
    const uint32_t KY = p->KY ? p->KY : 1;
    MUYO_REQUIRE(KY <= 65535u, "argmax: KY %u exceeds 65535", KY);
    const size_t need = muyo_cuda_argmax_workspace_size(p);
    MUYO_REQUIRE(workspace && workspace_bytes >= need, "argmax: workspace of %zu bytes needed, %zu given", need,
                 workspace_bytes);
    MUYO_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 7u) == 0, "argmax: workspace must be 8-byte aligned");
    return argmax_launch(a, p->KX, KY, 0, static_cast<ArgPair*>(workspace), d, as_stream(stream));
}

extern "C" int muyo_cuda_copy_f32(const MuyoUnaryParams* p, const float* a, float* d, void* stream)
{
    clear_error();
    MUYO_REQUIRE(p && a && d, "copy: null parameter block or buffer");
    const Dims4 S = dims(p->ne00, p->ne01, p->ne02, p->ne03, p->nb00, p->nb01, p->nb02, p->nb03);
    const Dims4 T = dims(p->ne10, p->ne11, p->ne12, p->ne13, p->nb10, p->nb11, p->nb12, p->nb13);
    MUYO_REQUIRE(p->ne > 0, "copy: ne must be positive");
    MUYO_REQUIRE((long long)p->ne <= count(S) && (long long)p->ne <= count(T),
                 "copy: ne exceeds the source or destination shape");
    MUYO_CUDA_TRY(launch_kernel(k_copy, dim3(grid_for(p->ne)), dim3(kThreads), 0, as_stream(stream), true, S, T, p->a_offset, p->d_offset, a, d, p->ne));
    MUYO_LAUNCH_CHECK();
    return MUYO_OK;
}

extern "C" int muyo_cuda_mat_vec_f16_argmax(const MuyoMatVecParams* p, const void* a, const float* b, float* d,
                                            uint32_t row_begin, void* pair_out, void* workspace,
                                            size_t workspace_bytes, void* stream)
{
    clear_error();
    MUYO_REQUIRE(p && pair_out, "mat_vec_argmax: null parameter block or pair output");
    MUYO_REQUIRE(p->batches <= 1, "mat_vec_argmax: one batch only");
    MUYO_REQUIRE(p->fusion_flags == 0, "mat_vec_argmax: no fusion flags");
    MUYO_REQUIRE((uint64_t)row_begin + p->rows <= (uint64_t)INT_MAX, "mat_vec_argmax: global row index overflows");
    MuyoGenericParams g{p->rows, 1, 0, 0, 0, 0};
    const size_t need = muyo_cuda_argmax_workspace_size(&g);
    MUYO_REQUIRE(workspace && workspace_bytes >= need, "mat_vec_argmax: workspace of %zu bytes needed, %zu given",
                 need, workspace_bytes);
    MUYO_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 7u) == 0 &&
                     (reinterpret_cast<uintptr_t>(pair_out) & 7u) == 0,
                 "mat_vec_argmax: workspace and pair_out must be 8-byte aligned");
    int rc = mat_vec_any(true, p, a, b, d, nullptr, nullptr, stream);
    if (rc != MUYO_OK)
        return rc;
    const cudaStream_t s = as_stream(stream);
    ArgPair* part = static_cast<ArgPair*>(workspace);
    rc = argmax_launch(d, p->rows, 1, (int)row_begin, part, nullptr, s);
    if (rc != MUYO_OK)
        return rc;
    // One shard pair: reduce the partials into pair_out.
    MUYO_CUDA_TRY(launch_kernel(k_pairs_to_pair, dim3(1), dim3(kThreads), 0, s, true, part, argmax_blocks(p->rows), static_cast<ArgPair*>(pair_out)));
    MUYO_LAUNCH_CHECK();
    return MUYO_OK;
}

extern "C" int muyo_cuda_argmax_pairs(const void* pairs, uint32_t n_pairs, int32_t* d, void* stream)
{
    clear_error();
    MUYO_REQUIRE(pairs && d && n_pairs > 0, "argmax_pairs: null buffer or no pairs");
    MUYO_REQUIRE((reinterpret_cast<uintptr_t>(pairs) & 7u) == 0, "argmax_pairs: pairs must be 8-byte aligned");
    MUYO_CUDA_TRY(launch_kernel(k_argmax_final, dim3(1), dim3(kThreads), 0, as_stream(stream), true, static_cast<const ArgPair*>(pairs), (int)n_pairs, d));
    MUYO_LAUNCH_CHECK();
    return MUYO_OK;
}

// ---- argmax without a caller workspace ---------------------------------------------------------
// For callers that cannot hand the library device memory: they run where allocating is off limits
// (a fixed memory budget already carved up by a pool, a latency-critical loop where cudaMalloc's
// implicit device synchronisation is unacceptable) or hold no device allocator at all (a thin FFI
// host that only passes logits in and reads an index back). The partial pairs live in a static
// device array compiled into this library, so the call itself allocates nothing.

namespace muyo {
constexpr int kNoAllocArgmaxPairs = 8192;  // 64 KB of (value, index) partials per device
static __device__ __align__(256) ArgPair g_noalloc_argmax_pairs[kNoAllocArgmaxPairs];
}  // namespace muyo

namespace {
constexpr int kMaxCachedDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[kMaxCachedDevices] = {};

// Device address of the static partials on the current device, resolved once per device.
int noalloc_scratch(ArgPair** out)
{
    int dev = -1;
    MUYO_CUDA_TRY(cudaGetDevice(&dev));
    MUYO_REQUIRE(dev >= 0 && dev < kMaxCachedDevices, "argmax_noalloc: device ordinal %d is not supported", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (!g_noalloc_ptr[dev]) {
        void* ptr = nullptr;
        MUYO_CUDA_TRY(cudaGetSymbolAddress(&ptr, muyo::g_noalloc_argmax_pairs));
        MUYO_REQUIRE(ptr != nullptr, "argmax_noalloc: no device address for the static scratch");
        g_noalloc_ptr[dev] = ptr;
    }
    *out = static_cast<ArgPair*>(g_noalloc_ptr[dev]);
    return MUYO_OK;
}
}  // namespace

extern "C" size_t muyo_cuda_argmax_noalloc_max_pairs(void) { return (size_t)kNoAllocArgmaxPairs; }

extern "C" int muyo_cuda_argmax_noalloc(const MuyoGenericParams* p, const float* a, int32_t* d, void* stream)
{
    clear_error();
    MUYO_REQUIRE(p && a && d, "argmax_noalloc: null parameter block or buffer");
    MUYO_REQUIRE(p->KX > 0 && p->KX <= (uint32_t)INT_MAX, "argmax_noalloc: KX must be in [1, INT_MAX]");
    const uint32_t KY = p->KY ? p->KY : 1;
    MUYO_REQUIRE(KY <= 65535u, "argmax_noalloc: KY %u exceeds 65535", KY);
    const uint64_t pairs = (uint64_t)KY * (uint64_t)argmax_blocks(p->KX);
    MUYO_REQUIRE(pairs <= (uint64_t)kNoAllocArgmaxPairs,
                 "argmax_noalloc: KY * ceil(KX / %d) = %llu partials exceeds the static scratch of %d; "
                 "use muyo_cuda_argmax with a workspace",
                 kArgmaxChunk, (unsigned long long)pairs, kNoAllocArgmaxPairs);
    ArgPair* part = nullptr;
    const int rc = noalloc_scratch(&part);
    if (rc != MUYO_OK)
        return rc;
    // Every partial is written by the first kernel before the second reads it, so no part of the
    // scratch has to start at zero.
    return argmax_launch(a, p->KX, KY, 0, part, d, as_stream(stream));
}


// ---- row-sharded GEMV + all-gather over NVLink: host side -------------------------------------------
struct MuyoP2PGroup {
    int device = -1, world = 0, rank = 0;
    uint32_t rows_total = 0;
    char* buf = nullptr;                 // own buffer: header, then the output
    void* peer[kP2PMaxRanks] = {};       // opened peer buffers (nullptr for this rank)
    ArgPair* cta_pairs = nullptr;        // per-CTA scratch (local)
    int max_ctas = 0;
    uint32_t epoch = 0;                  // calls issued through muyo_cuda_mat_vec_f16_allgather (not replays)
    bool dead = false;                   // a call timed out: the ranks' epochs no longer agree
};

// Header, then two output slots (call epoch e uses slot e & 1), each 256-byte aligned.
static size_t p2p_slot_bytes(uint32_t rows_total) { return ((size_t)rows_total * sizeof(float) + 255) / 256 * 256; }
static size_t p2p_bytes(uint32_t rows_total) { return sizeof(P2PHeader) + 2 * p2p_slot_bytes(rows_total); }
static float* p2p_slot(char* base, uint32_t rows_total, uint32_t epoch)
{
    return reinterpret_cast<float*>(base + sizeof(P2PHeader) + (epoch & 1) * p2p_slot_bytes(rows_total));
}

extern "C" size_t muyo_p2p_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int muyo_p2p_create(int world, int rank, uint32_t rows_total, MuyoP2PGroup** out, void* handle_out)
{
    clear_error();
    MUYO_REQUIRE(out && handle_out, "p2p_create: null argument");
    MUYO_REQUIRE(world >= 1 && world <= kP2PMaxRanks && rank >= 0 && rank < world,
                 "p2p_create: world %d / rank %d outside 1..%d", world, rank, kP2PMaxRanks);
    MUYO_REQUIRE(rows_total > 0 && rows_total <= (uint32_t)INT_MAX, "p2p_create: rows_total must be positive");
    MuyoP2PGroup* g = new (std::nothrow) MuyoP2PGroup;
    if (!g) {
        set_error("p2p_create: out of host memory");
        return MUYO_ENOMEM;
    }
    g->world = world, g->rank = rank, g->rows_total = rows_total;
    int rc = MUYO_OK;
    do {
        if (cudaGetDevice(&g->device) != cudaSuccess) { rc = MUYO_ECUDA; break; }
        g->max_ctas = sm_count() * 8;
        if (cudaMalloc(&g->buf, p2p_bytes(rows_total)) != cudaSuccess ||
            cudaMalloc(&g->cta_pairs, sizeof(ArgPair) * (size_t)g->max_ctas) != cudaSuccess) {
            rc = MUYO_ENOMEM;
            break;
        }
        if (cudaMemset(g->buf, 0, p2p_bytes(rows_total)) != cudaSuccess ||
            cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle_out), g->buf) != cudaSuccess ||
            cudaDeviceSynchronize() != cudaSuccess) {
            rc = MUYO_ECUDA;
            break;
        }
    } while (0);
    if (rc != MUYO_OK) {
        set_error("p2p_create: device allocation or IPC handle failed (%s)", cudaGetErrorString(cudaGetLastError()));
        cudaFree(g->buf);
        cudaFree(g->cta_pairs);
        delete g;
        return rc;
    }
    *out = g;
    return MUYO_OK;
}

extern "C" int muyo_p2p_connect(MuyoP2PGroup* g, const void* handles)
{
    clear_error();
    MUYO_REQUIRE(g && handles, "p2p_connect: null argument");
    const cudaIpcMemHandle_t* h = static_cast<const cudaIpcMemHandle_t*>(handles);
    for (int r = 0; r < g->world; ++r) {
        if (r == g->rank || g->peer[r])
            continue;
        MUYO_CUDA_TRY(cudaIpcOpenMemHandle(&g->peer[r], h[r], cudaIpcMemLazyEnablePeerAccess));
    }
    return MUYO_OK;
}

extern "C" int muyo_p2p_output(MuyoP2PGroup* g, float** y)
{
    clear_error();
    MUYO_REQUIRE(g && y, "p2p_output: null argument");
    *y = p2p_slot(g->buf, g->rows_total, g->epoch);
    return MUYO_OK;
}

extern "C" int muyo_p2p_check(MuyoP2PGroup* g)
{
    clear_error();
    MUYO_REQUIRE(g, "p2p_check: null group");
    int e = 0;
    MUYO_CUDA_TRY(cudaMemcpy(&e, g->buf + offsetof(P2PHeader, err), sizeof(int), cudaMemcpyDeviceToHost));
    if (e) {
        MUYO_CUDA_TRY(cudaMemset(g->buf + offsetof(P2PHeader, err), 0, sizeof(int)));
        g->dead = true;
        set_error("p2p: a wait for a peer's flag expired (a rank did not take part in the call); the group must be "
                  "destroyed and created again on every rank");
        return MUYO_ETIMEOUT;
    }
    return MUYO_OK;
}

extern "C" int muyo_cuda_mat_vec_f16_allgather(MuyoP2PGroup* g, const MuyoMatVecParams* p, const void* a,
                                               const float* b, uint32_t row_begin, int32_t* token, void* stream)
{
    clear_error();
    MUYO_REQUIRE(g && token, "mat_vec_allgather: null group or token");
    if (g->dead) {
        set_error("mat_vec_allgather: an earlier call of this group timed out; destroy it and create a new one on "
                  "every rank");
        return MUYO_ESTATE;
    }
    for (int r = 0; r < g->world; ++r)
        MUYO_REQUIRE(r == g->rank || g->peer[r], "mat_vec_allgather: rank %d is not connected", r);
    MUYO_REQUIRE(p && (p->batches <= 1) && p->fusion_flags == 0, "mat_vec_allgather: one batch, no fusion flags");
    MUYO_REQUIRE((uint64_t)row_begin + p->rows <= g->rows_total, "mat_vec_allgather: rows [%u, %u) exceed %u", row_begin,
                 row_begin + p->rows, g->rows_total);
    MatVecDev q{};
    if (p->rows == 0) {
        // An empty shard (more ranks than rows): the rank still takes part in the exchange, with a
        // pair that never wins; A is not read.
        MUYO_REQUIRE(b && p->ncols > 0 && p->ncols <= (uint32_t)kMaxStagedK, "mat_vec_allgather: ncols %u outside 1..%d",
                     p->ncols, kMaxStagedK);
        q.ncols = (int)p->ncols;
        q.rows = 0;
        q.stride_a = q.ncols;
        q.k8 = q.ncols / 8;
    } else {
        int rc = mat_vec_prepare(p, a, b, reinterpret_cast<float*>(g->buf), nullptr, nullptr, 2, q);
        if (rc != MUYO_OK)
            return rc;
    }
    MUYO_REQUIRE(q.k8 > 0 && aligned16(b), "mat_vec_allgather: A and x must be 16-byte aligned with rows a multiple of 8");
    P2PArgs args{};
    args.A = static_cast<const __half*>(a);
    args.x = b;
    args.K = q.ncols, args.k8 = q.k8, args.local_rows = q.rows, args.row_begin = (int)row_begin;
    args.rows_total = (int)g->rows_total, args.world = g->world, args.rank = g->rank, args.lda = q.stride_a;
    args.slot_floats = (long long)(p2p_slot_bytes(g->rows_total) / sizeof(float));
    ++g->epoch;
    for (int r = 0; r < g->world; ++r) {
        char* base = r == g->rank ? g->buf : static_cast<char*>(g->peer[r]);
        args.hdr[r] = reinterpret_cast<P2PHeader*>(base);
        args.y[r] = p2p_slot(base, g->rows_total, 0);
    }
    args.cta_pairs = g->cta_pairs;
    args.token = token;
    // The tile shape of muyo_cuda_mat_vec_f16 for the same shard (bit-identical values); the grid is what
    // is resident at once, each CTA taking a contiguous range of tiles.
    const bool two_rows = mat_vec_two_rows(q);
    const int ksplit = mat_vec_ksplit(q, 1, two_rows ? 2 : 1);
    const bool u8 = q.k8 / ksplit / 32 >= 8;
    auto k = k_gemv_allgather<1, 4, 1>;
#define MUYO_P2P_PICK(R)                                                                          \
    k = ksplit == 4 ? (u8 ? k_gemv_allgather<R, 8, 4> : k_gemv_allgather<R, 4, 4>)                \
                    : ksplit == 2 ? (u8 ? k_gemv_allgather<R, 8, 2> : k_gemv_allgather<R, 4, 2>)  \
                                  : (u8 ? k_gemv_allgather<R, 8, 1> : k_gemv_allgather<R, 4, 1>)
    if (two_rows)
        MUYO_P2P_PICK(2);
    else
        MUYO_P2P_PICK(1);
#undef MUYO_P2P_PICK
    const int tile_rows = 8 / ksplit * (two_rows ? 2 : 1);
    const int ntiles = (q.rows + tile_rows - 1) / tile_rows;
    const size_t smem = (size_t)q.ncols * sizeof(float);
    MUYO_CUDA_TRY(set_smem(k, smem));
    int per_sm = 0;
    MUYO_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kThreads, smem));
    int grid = per_sm > 0 ? per_sm * sm_count() : 1;
    if (grid > g->max_ctas)
        grid = g->max_ctas;
    if (grid > ntiles)
        grid = ntiles > 0 ? ntiles : 1;  // an empty shard runs one CTA: the exchange alone
    const cudaStream_t s = as_stream(stream);
    MUYO_CUDA_TRY(launch_kernel(k, dim3(grid), dim3(kThreads), smem, s, true, args));
    MUYO_LAUNCH_CHECK();
    return MUYO_OK;
}

extern "C" int muyo_p2p_destroy(MuyoP2PGroup* g)
{
    clear_error();
    if (!g)
        return MUYO_OK;
    cudaSetDevice(g->device);
    cudaDeviceSynchronize();
    for (int r = 0; r < kP2PMaxRanks; ++r)
        if (g->peer[r])
            cudaIpcCloseMemHandle(g->peer[r]);
    cudaFree(g->buf);
    cudaFree(g->cta_pairs);
    delete g;
    return MUYO_OK;
}
