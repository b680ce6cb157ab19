// The batch-1 F16-weight GEMV core: y = W x, W F16 row-major [rows][K], x F32, FP32 accumulate.
//
// The GEMV moves 2 bytes of weight per multiply-add, so it is bound by HBM, not by the tensor
// cores: it issues no MMA. Instead each warp streams ROWS rows (of NMAT matrices sharing x) with
// 16-byte loads, U of them per row in flight per lane, L1 bypassed. Lane l takes the 8-column
// chunks l, l+32, l+64, ... of each row, so one warp instruction reads 512 contiguous bytes of a row.
// x is staged in shared memory once per CTA in a split layout (first halves of every chunk, then
// second halves) so that the 32 lanes of a warp read 32 consecutive 16-byte words: no bank
// conflicts. The per-lane sums are combined with a butterfly of shuffles.
#pragma once

#include "common.cuh"

namespace muyo {

// Shared-memory layout of a staged K-vector: element k = 8c + j lives at
//   lo[c*4 + j]           for j < 4
//   lo[K8*4 + c*4 + j-4]  for j >= 4
// The tail k >= 8*K8 (K not a multiple of 8) is stored after both halves, at 8*K8 + (k - 8*K8).
__device__ __forceinline__ int xs_index(int k, int K8)
{
    const int c = k >> 3, j = k & 7;
    if (c >= K8)
        return k;  // tail: 8*K8 + (k - 8*K8)
    return j < 4 ? c * 4 + j : K8 * 4 + c * 4 + (j - 4);
}

// float4 q of a K-vector (elements 4q .. 4q+3) in the split layout above, as a float4 index: the
// first half of chunk q/2 when q is even, the second half when q is odd.
__device__ __forceinline__ int xs_slot4(int q, int K8) { return (q & 1) ? K8 + (q >> 1) : (q >> 1); }

// Asks L2 to start fetching `bytes` (a multiple of 16) from the 16-byte-aligned global address p;
// no registers or shared memory are involved and the call does not wait.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes)
{
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Rows [row0, row0 + nrows) of a row-major F16 matrix with row stride ldw elements (ldw % 8 == 0),
// prefetched to L2 in pieces of at most 64 KB.
__device__ __forceinline__ void prefetch_rows_l2(const __half* w, size_t ldw, int row0, int nrows)
{
    const char* p = reinterpret_cast<const char*>(w + (size_t)row0 * ldw);
    size_t left = (size_t)nrows * ldw * sizeof(__half);
    while (left > 0) {
        const uint32_t n = left > 65536 ? 65536u : (uint32_t)left;
        prefetch_l2(p, n);
        p += n;
        left -= n;
    }
}

// s + w[0..7] . (xa, xb): one 16-byte chunk of F16 weights against its 8 staged x values, in a
// fixed order (every GEMV path here uses it, so their sums agree bit for bit).
__device__ __forceinline__ float dot_chunk(uint4 w, float4 xa, float4 xb, float s)
{
    float2 f = h2_to_f2(w.x);
    s = fmaf(f.x, xa.x, s);
    s = fmaf(f.y, xa.y, s);
    f = h2_to_f2(w.y);
    s = fmaf(f.x, xa.z, s);
    s = fmaf(f.y, xa.w, s);
    f = h2_to_f2(w.z);
    s = fmaf(f.x, xb.x, s);
    s = fmaf(f.y, xb.y, s);
    f = h2_to_f2(w.w);
    s = fmaf(f.x, xb.z, s);
    s = fmaf(f.y, xb.w, s);
    return s;
}

template <int ROWS, int U, int NMAT>
struct GemvArgs {
    const __half* w[NMAT];
    size_t ldw;  // row stride in elements (multiple of 8 for the vector path)
};

// acc[m][r] += sum over this lane's chunks c in [c_begin, c_end) of W_m[row0 + r][8c .. 8c+7] .
// x[8c .. 8c+7], for r < ROWS (rows >= nvalid are read from row0, and their sums must be ignored by
// the caller). K8 is the staged vector's chunk count (its shared-memory layout).
template <int ROWS, int U, int NMAT>
__device__ __forceinline__ void warp_gemv_f16_range(const GemvArgs<ROWS, U, NMAT>& a, int row0, int nvalid,
                                                    const float* __restrict__ xs, int K8, int c_begin, int c_end,
                                                    int lane, float (&acc)[NMAT][ROWS])
{
    const float4* xlo = reinterpret_cast<const float4*>(xs);
    const float4* xhi = reinterpret_cast<const float4*>(xs + 4 * K8);
    const uint4* rowp[NMAT][ROWS];
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
            const int rr = r < nvalid ? r : 0;
            rowp[m][r] = reinterpret_cast<const uint4*>(a.w[m] + (size_t)(row0 + rr) * a.ldw);
        }

    for (int base = c_begin; base < c_end; base += WARP * U) {
        uint4 wv[NMAT][ROWS][U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = base + lane + WARP * u;
            const bool ok = c < c_end;
#pragma unroll
            for (int m = 0; m < NMAT; ++m)
#pragma unroll
                for (int r = 0; r < ROWS; ++r)
                    wv[m][r][u] = ok ? ld_stream16(rowp[m][r] + c) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = base + lane + WARP * u;
            if (c < c_end) {
                const float4 xa = xlo[c];
                const float4 xb = xhi[c];
#pragma unroll
                for (int m = 0; m < NMAT; ++m)
#pragma unroll
                    for (int r = 0; r < ROWS; ++r)
                        acc[m][r] = dot_chunk(wv[m][r][u], xa, xb, acc[m][r]);
            }
        }
    }
}

__device__ __forceinline__ uint4 lds16(unsigned addr)
{
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(addr));
    return r;
}

// As warp_gemv_f16_range, with the weight rows already in shared memory: matrix m's row lrow0 + r
// starts at shared address wsm[m] + (lrow0 + r) * row_bytes (rows of K8 16-byte chunks). The
// products are accumulated in the same order, so the sums are bit-identical.
template <int ROWS, int U, int NMAT>
__device__ __forceinline__ void warp_gemv_f16_smem(const unsigned (&wsm)[NMAT], unsigned row_bytes, int lrow0,
                                                   int nvalid, const float* __restrict__ xs, int K8, int c_begin,
                                                   int c_end, int lane, float (&acc)[NMAT][ROWS])
{
    const float4* xlo = reinterpret_cast<const float4*>(xs);
    const float4* xhi = reinterpret_cast<const float4*>(xs + 4 * K8);
    unsigned rowa[NMAT][ROWS];
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int r = 0; r < ROWS; ++r)
            rowa[m][r] = wsm[m] + (unsigned)(lrow0 + (r < nvalid ? r : 0)) * row_bytes;
    for (int base = c_begin; base < c_end; base += WARP * U) {
        uint4 wv[NMAT][ROWS][U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = base + lane + WARP * u;
            const bool ok = c < c_end;
#pragma unroll
            for (int m = 0; m < NMAT; ++m)
#pragma unroll
                for (int r = 0; r < ROWS; ++r)
                    wv[m][r][u] = ok ? lds16(rowa[m][r] + 16u * (unsigned)c) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = base + lane + WARP * u;
            if (c < c_end) {
                const float4 xa = xlo[c];
                const float4 xb = xhi[c];
#pragma unroll
                for (int m = 0; m < NMAT; ++m)
#pragma unroll
                    for (int r = 0; r < ROWS; ++r)
                        acc[m][r] = dot_chunk(wv[m][r][u], xa, xb, acc[m][r]);
            }
        }
    }
}

template <int ROWS, int U, int NMAT>
__device__ __forceinline__ void warp_gemv_f16(const GemvArgs<ROWS, U, NMAT>& a, int row0, int nvalid,
                                              const float* __restrict__ xs, int K8, int lane,
                                              float (&acc)[NMAT][ROWS])
{
    warp_gemv_f16_range<ROWS, U, NMAT>(a, row0, nvalid, xs, K8, 0, K8, lane, acc);
}

// Columns 8*K8 .. K-1 when K is not a multiple of 8 (scalar loads; the rows must then be read
// through the scalar path, see mat_vec_f16 in ops.cu).
template <int ROWS, int NMAT>
__device__ __forceinline__ void warp_gemv_f16_tail(const __half* const* w, size_t ldw, int row0, int nvalid,
                                                   const float* __restrict__ xs, int K8, int K, int lane,
                                                   float (&acc)[NMAT][ROWS])
{
    for (int k = 8 * K8 + lane; k < K; k += WARP) {
        const float xk = xs[k];
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
            for (int r = 0; r < ROWS; ++r) {
                const int rr = r < nvalid ? r : 0;
                acc[m][r] = fmaf(__half2float(w[m][(size_t)(row0 + rr) * ldw + k]), xk, acc[m][r]);
            }
    }
}

template <int ROWS, int NMAT>
__device__ __forceinline__ void warp_reduce_acc(float (&acc)[NMAT][ROWS])
{
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int r = 0; r < ROWS; ++r)
            acc[m][r] = warp_sum(acc[m][r]);
}

}  // namespace muyo
