// On-device token sampler: Sampler::Sample (src/Sampler.cpp:10-98) with its std::mt19937_64 stream
// kept in device memory, so that non-greedy decoding needs no host round trip.
//
// One thread-block cluster of C = 8 (or 16) CTAs of 1024 threads. CTA r owns the contiguous logits
// [r*S, (r+1)*S) and holds them in shared memory: the row is read from L2 once, and every pass
// after that runs on the shared memory of C SMs, the CTAs exchanging histograms and counts through
// distributed shared memory. In the reference's order:
//   1. repetition penalty: each CTA counts the history window's occurrences of its own ids and
//      applies the penalty that many times to each id's logit, which is what the reference's
//      in-order loop does to it (one id's updates are sequential on its own value; ids are
//      independent);
//   2. temperature <= 0: the first index of the maximum (CTA argmax, then rank 0 over the CTAs);
//   3. logits /= temperature (written back: logits are modified in place, as the reference does);
//   4. top-k: a radix select of the k-th largest key, digits of 11, 11 and 10 bits from the top;
//      per-CTA histograms with warp-aggregated shared atomics, summed across the cluster. The
//      candidates (keys above the threshold, and the lowest-index keys equal to it) go to rank 0 in
//      index order, which sorts them by (logit descending, index ascending);
//   5. rank 0: weights exp(double(l_i - l_0)) and their quotients by the total in parallel; one
//      thread forms the sums in order (double), the nucleus cut, draws u = canonical double from the
//      engine and picks the token.
// mt19937_64 is restated from its published definition (Matsumoto & Nishimura): n = 312, m = 156,
// r = 31, a = 0xB5026F5AA96619E9, tempering (29, 0x5555555555555555), (17, 0x71D67FFFEDA60000),
// (37, 0xFFF7EEE000000000), 43; seeding multiplier 6364136223846793005. The state refill runs in
// shared memory in three parallel phases that equal the sequential recurrence.
#include <cooperative_groups.h>

#include <climits>
#include <cmath>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace muyo {

constexpr int kSampleThreads = 1024;
constexpr int kSampleMaxK = 4096;
constexpr int kHistBins = 2048;    // radix digits of 11, 11 and 10 bits
constexpr int kRankSortMax = 128;  // rank 0 orders up to this many candidates by counting, more by a bitonic sort
constexpr int kSmemMax = 223 * 1024;  // dynamic; the 227 KB per CTA also hold the static arrays (< 4 KB)

struct Mt64State {
    unsigned long long mt[312];
    int idx;
    int pad;
};

__global__ void k_mt64_seed(Mt64State* s, unsigned long long seed)
{
    s->mt[0] = seed;
    for (int i = 1; i < 312; ++i)
        s->mt[i] = 6364136223846793005ULL * (s->mt[i - 1] ^ (s->mt[i - 1] >> 62)) + (unsigned long long)i;
    s->idx = 312;
}

// One step of the recurrence: word i from words i (upper bit), i + 1 (lower bits) and i + m.
__device__ __forceinline__ unsigned long long mt64_twist(unsigned long long cur, unsigned long long next,
                                                         unsigned long long far)
{
    const unsigned long long x = (cur & 0xFFFFFFFF80000000ULL) | (next & 0x7FFFFFFFULL);
    return far ^ (x >> 1) ^ ((x & 1ULL) ? 0xB5026F5AA96619E9ULL : 0ULL);
}

__device__ __forceinline__ unsigned long long mt64_temper(unsigned long long y)
{
    y ^= (y >> 29) & 0x5555555555555555ULL;
    y ^= (y << 17) & 0x71D67FFFEDA60000ULL;
    y ^= (y << 37) & 0xFFF7EEE000000000ULL;
    return y ^ (y >> 43);
}

// Order-preserving unsigned key of a float (ascending); -0 is folded onto +0, which compares equal.
__device__ __forceinline__ unsigned sort_key(float f)
{
    unsigned b = __float_as_uint(f);
    if (b == 0x80000000u)
        b = 0u;
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float key_value(unsigned k)
{
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// Block exclusive scan of one int per thread (kSampleThreads threads); returns the total.
__device__ int block_exclusive_scan(int v, int& excl, int* warp_sums)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o)
            x += y;
    }
    if (lane == 31)
        warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = lane < kSampleThreads / 32 ? warp_sums[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o)
                w += y;
        }
        warp_sums[lane] = w;  // inclusive prefix over warps
    }
    __syncthreads();
    excl = x - v + (warp > 0 ? warp_sums[warp - 1] : 0);
    const int total = warp_sums[kSampleThreads / 32 - 1];
    __syncthreads();
    return total;
}

// Left-to-right double sum of x[0, n) (the reference's loop order), loads issued eight at a time;
// pre[j] receives every running sum x[0] + ... + x[j].
__device__ double ordered_prefix(const double* __restrict__ x, double* __restrict__ pre, int n)
{
    double s = 0.0;
    int j = 0;
    for (; j + 8 <= n; j += 8) {
        double t[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
            t[u] = x[j + u];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            s += t[u];
            pre[j + u] = s;
        }
    }
    for (; j < n; ++j) {
        s += x[j];
        pre[j] = s;
    }
    return s;
}

// First j whose left-to-right prefix sum x[0] + ... + x[j] is >= target; n if none.
__device__ int first_reaching(const double* x, int n, double target)
{
    double s = 0.0;
    for (int j = 0; j < n; j += 8) {
        double t[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
            t[u] = j + u < n ? x[j + u] : 0.0;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            if (j + u < n) {
                s += t[u];
                if (s >= target)
                    return j + u;
            }
        }
    }
    return n;
}

// (key descending, id ascending): a before b
__device__ __forceinline__ bool cand_before(unsigned ka, int ia, unsigned kb, int ib)
{
    return ka > kb || (ka == kb && ia < ib);
}

// One bitonic stage between register slots r and r | RS of each thread (entries r * T + tid).
template <int E, int RS>
__device__ __forceinline__ void slot_stage(unsigned (&k)[E], int (&ix)[E], int size, int T)
{
    if constexpr (RS < E) {
#pragma unroll
        for (int r = 0; r < E; ++r) {
            if ((r & RS) == 0) {
                const int r2 = r | RS, j = r * T + (int)threadIdx.x;
                const bool desc = (j & size) == 0;
                if (cand_before(k[r], ix[r], k[r2], ix[r2]) != desc) {
                    const unsigned tk = k[r];
                    const int ti = ix[r];
                    k[r] = k[r2], ix[r] = ix[r2];
                    k[r2] = tk, ix[r2] = ti;
                }
            }
        }
    }
}

// Bitonic sort of keys/idx[0, P) in shared memory by cand_before, P a power of two in [256, 8192]:
// thread t holds the E = P / T entries t, t + T, ... (T = min(P, block threads)) in registers.
// Partners closer than 32 are exchanged by warp shuffles, partners a multiple of T apart are in the
// same thread, and only the strides in between go through shared memory.
template <int E>
__device__ void bitonic_sort_regs(unsigned* keys, int* idx, int P)
{
    const int tid = threadIdx.x;
    const int T = E > 1 ? kSampleThreads : P;
    const bool active = tid < T;
    unsigned k[E];
    int ix[E];
#pragma unroll
    for (int r = 0; r < E; ++r) {
        k[r] = active ? keys[r * T + tid] : 0u;
        ix[r] = active ? idx[r * T + tid] : INT_MAX;
    }
    for (int size = 2; size <= P; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride >= T) {  // within this thread (E > 1): slots r and r + stride / T
                const int rs = stride / T;
                if (rs == 1)
                    slot_stage<E, 1>(k, ix, size, T);
                else if (rs == 2)
                    slot_stage<E, 2>(k, ix, size, T);
                else
                    slot_stage<E, 4>(k, ix, size, T);
            } else {
                const bool via_smem = stride >= 32;
                if (via_smem) {
                    __syncthreads();
                    if (active) {
#pragma unroll
                        for (int r = 0; r < E; ++r)
                            keys[r * T + tid] = k[r], idx[r * T + tid] = ix[r];
                    }
                    __syncthreads();
                }
                if (active) {
#pragma unroll
                    for (int r = 0; r < E; ++r) {
                        const int j = r * T + tid;
                        unsigned pk;
                        int pi;
                        if (via_smem) {
                            pk = keys[j ^ stride];
                            pi = idx[j ^ stride];
                        } else {
                            pk = __shfl_xor_sync(0xffffffffu, k[r], stride);
                            pi = __shfl_xor_sync(0xffffffffu, ix[r], stride);
                        }
                        // the lower entry of a descending pair keeps the earlier candidate
                        const bool take_first = ((j & stride) == 0) == ((j & size) == 0);
                        if (cand_before(pk, pi, k[r], ix[r]) == take_first)
                            k[r] = pk, ix[r] = pi;
                    }
                }
            }
        }
    }
    __syncthreads();
    if (active) {
#pragma unroll
        for (int r = 0; r < E; ++r)
            keys[r * T + tid] = k[r], idx[r * T + tid] = ix[r];
    }
    __syncthreads();
}

struct SampleArgs {
    float temperature;
    int top_k;
    float top_p;
    float repeat_penalty;
    int repeat_last_n;
    int vocab;
    float* logits;
    const int32_t* history;
    int hist_len;
    Mt64State* rng;
    int32_t* token;
    // Decode-graph mode (gate != nullptr): gate = {step, prompt_end, total} of the model's control
    // block, read after the LM head advanced step to n. The sampler runs only for a generated
    // position (prompt_end <= n < total, n < max_seq), with history = tokens[0, n) (every id in the
    // cache) and the id also stored at tokens[n]; otherwise it returns without drawing.
    const int32_t* gate;
    int32_t* tokens;
    int max_seq;
    int slice;     // logits per CTA (a multiple of 4, below 2^16)
    int cand_off;  // dynamic shared memory: [0, cand_off) the CTA's keys, then the penalty counts
    int hist_off;  // (later rank 0's candidates), then five radix histograms
    int cap;       // rank 0's gather buffer: entries (a power of two >= k)
};

struct SampleSmem {
    int cand_off, hist_off, bytes, cap;
};

__host__ __device__ inline int sample_pow2(int k)
{
    int p = 1;
    while (p < k)
        p <<= 1;
    return p;
}

// Dynamic shared memory of one CTA for a slice of `slice` logits, k candidates and a gather
// buffer of `cap` entries: keys, then the penalty counts or rank 0's candidates (gather buffer,
// sorted top-k of at most kRankSortMax entries, weights, quotients, prefix sums), then the histograms.
__host__ __device__ inline SampleSmem sample_smem(int slice, int k, int cap)
{
    const int counts = (slice + 1) / 2 * 4;  // 16-bit occurrence counts, two per word
    const int sk = sample_pow2(k) < kRankSortMax ? sample_pow2(k) : kRankSortMax;
    const int cand = 8 * cap + 8 * sk + 24 * k;
    SampleSmem m;
    m.cap = cap;
    m.cand_off = slice * 4;
    m.hist_off = m.cand_off + ((counts > cand ? counts : cand) + 15) / 16 * 16;
    m.bytes = m.hist_off + 5 * kHistBins * 4;
    return m;
}

__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// Adds one to bins[d] for every active lane, one atomic per distinct d in the warp.
__device__ __forceinline__ void warp_count(unsigned* bins, unsigned d, int lane)
{
    const unsigned grp = __match_any_sync(__activemask(), d);
    if (lane == __ffs(grp) - 1)
        atomicAdd(&bins[d], (unsigned)__popc(grp));
}

// Appends (key, id) to rank 0's buffers for every active lane with `take`, one slot reservation per
// warp; the order of the entries is arbitrary.
__device__ __forceinline__ void warp_append(bool take, unsigned key, int id, int* slots, unsigned* keys, int* ids,
                                            int lane)
{
    const unsigned act = __activemask();
    const unsigned b = __ballot_sync(act, take);
    if (b == 0u)
        return;
    const int leader = __ffs(b) - 1;
    int at = 0;
    if (lane == leader)
        at = atomicAdd(slots, __popc(b));
    at = __shfl_sync(act, at, leader);
    if (take) {
        at += __popc(b & ((1u << lane) - 1u));
        keys[at] = key;
        ids[at] = id;
    }
}

__global__ void __launch_bounds__(kSampleThreads, 1) k_sample(SampleArgs a)
{
    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned* keys_loc = reinterpret_cast<unsigned*>(smem_raw);  // sort keys of this CTA's logits
    unsigned* cnt = reinterpret_cast<unsigned*>(smem_raw + a.cand_off);
    // radix histograms: four cluster-wide ones in rank 0 (pass 0, the full pass 0, passes 1 and 2)
    // and each CTA's own counts of the current pass
    unsigned* hist = reinterpret_cast<unsigned*>(smem_raw + a.hist_off);
    unsigned* hloc = hist + 4 * kHistBins;
    // rank 0's candidates: a gather buffer of a.cap (key, id) entries, then the sorted top-k
    unsigned* gkeys = reinterpret_cast<unsigned*>(smem_raw + a.cand_off);
    int* gidx = reinterpret_cast<int*>(gkeys + a.cap);
    __shared__ int warp_sums[32];
    __shared__ float sv[32];
    __shared__ int si[32];
    __shared__ unsigned sh_prefix;
    __shared__ int sh_remaining;
    __shared__ int sh_digit_count;  // keys (cluster-wide) with the selected prefix
    __shared__ int sh_gathered;     // keys (cluster-wide) with the selected pass-0 digit or a larger one
    __shared__ int sh_slots;        // rank 0: candidate slots handed out
    __shared__ int sh_lo;           // this CTA's lowest pass-0 digit counted
    __shared__ int sh_lo_max;       // the largest of the cluster's sh_lo
    __shared__ int sh_tot[2];       // this CTA's keys above / equal to the threshold
    __shared__ int sh_offs[3];      // above in lower ranks, equal in lower ranks, above in all ranks
    __shared__ int sh_hit;
    __shared__ unsigned long long mt[312];
    __shared__ int mt_idx;
    __shared__ double sh_total;
    pdl_wait();
    pdl_trigger();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rank = (int)cluster.block_rank(), C = (int)cluster.num_blocks();
    const int V = a.vocab, S = a.slice, base = rank * S;
    const int nloc = max(0, min(S, V - base));
    int hist_len = a.hist_len;
    const int32_t* history = a.history;
    int n = 0;
    if (a.gate) {  // uniform over the cluster: every thread reads the same words
        n = __ldcg(a.gate);
        if (n < __ldcg(a.gate + 1) || n >= __ldcg(a.gate + 2) || n >= a.max_seq)
            return;
        hist_len = n;
        history = a.tokens;
    }
    const bool temp = a.temperature > 0.0f;
    const bool pen = a.repeat_penalty != 1.0f && hist_len > 0;
    if (temp) {
        if (rank == 0) {
            for (int w = tid; w < 4 * kHistBins; w += kSampleThreads)
                hist[w] = 0u;
            if (tid == 0)
                sh_slots = 0;
            for (int j = tid; j < 312; j += kSampleThreads)  // the engine, used at the end
                mt[j] = a.rng->mt[j];
            if (tid == 0)
                mt_idx = a.rng->idx, sh_hit = INT_MAX;
        }
        cluster_arrive();  // completed by cluster_wait before the first count into rank 0
    }

    // 1. occurrences of this CTA's ids in the penalty window
    if (pen) {
        for (int w = tid; w < (nloc + 1) / 2; w += kSampleThreads)
            cnt[w] = 0u;
        __syncthreads();
        int begin = 0;
        if (a.repeat_last_n >= 0 && a.repeat_last_n < hist_len)
            begin = hist_len - a.repeat_last_n;
        for (int j = begin + tid; j < hist_len; j += kSampleThreads) {
            const int t = history[j] - base;
            if (t >= 0 && t < nloc)
                atomicAdd(&cnt[t >> 1], 1u << ((t & 1) * 16));
        }
        __syncthreads();
    }

    // 2-3. penalised (and temperature-scaled) logits, as keys in shared memory; eight loads in flight
    float bv = -INFINITY;
    int bi = INT_MAX;
    unsigned kmax = 0u;
    for (int j0 = tid; j0 < nloc; j0 += 8 * kSampleThreads) {
        float v8[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int j = j0 + u * kSampleThreads;
            v8[u] = j < nloc ? a.logits[base + j] : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int j = j0 + u * kSampleThreads;
            if (j >= nloc)
                break;
            float v = v8[u];
            bool changed = temp;
            if (pen) {
                unsigned c = (cnt[j >> 1] >> ((j & 1) * 16)) & 0xFFFFu;
                changed |= c != 0u;
                for (; c != 0u; --c)
                    v = v > 0.0f ? __fdiv_rn(v, a.repeat_penalty) : v * a.repeat_penalty;
            }
            if (temp)
                v = __fdiv_rn(v, a.temperature);
            if (changed)
                a.logits[base + j] = v;
            const unsigned key = sort_key(v);
            keys_loc[j] = key;
            kmax = max(kmax, key);
            if (pair_better(v, base + j, bv, bi))
                bv = v, bi = base + j;
        }
    }

    if (!temp) {  // greedy: the first index of the maximum
        warp_argmax(bv, bi);
        if (lane == 0)
            sv[warp] = bv, si[warp] = bi;
        __syncthreads();
        if (warp == 0) {
            bv = sv[lane], bi = si[lane];
            warp_argmax(bv, bi);
        }
        __syncthreads();
        if (tid == 0)
            sv[0] = bv, si[0] = bi;
        cluster.sync();
        if (rank == 0 && tid == 0) {
            for (int r = 1; r < C; ++r) {
                const float rv = *cluster.map_shared_rank(&sv[0], r);
                const int ri = *cluster.map_shared_rank(&si[0], r);
                if (pair_better(rv, ri, bv, bi))
                    bv = rv, bi = ri;
            }
            const int tok = bi == INT_MAX ? 0 : bi;
            *a.token = tok;
            if (a.gate)
                a.tokens[n] = tok;
        }
        cluster.sync();  // the other CTAs' shared memory stays live until rank 0 has read it
        return;
    }

    // 4. the k-th largest key. Radix digits [21, 32), [10, 21), [0, 10) of the sort key, counted
    // into rank 0's histograms. Pass 0 counts, in each CTA, only the digits from 4 below its largest
    // key's digit (one octave of magnitude); the cluster's counts are exact for every digit >= the
    // largest of those bounds, and when fewer than k keys lie there a full pass 0 runs. When the
    // keys in or above the selected pass-0 digit fit rank 0's gather buffer, they all go there and
    // rank 0 finishes alone; otherwise passes 1 and 2 run over the cluster.
    const int k = a.top_k <= 0 ? V : min(a.top_k, V);
    kmax = __reduce_max_sync(0xffffffffu, kmax);
    if (lane == 0)
        warp_sums[warp] = (int)(kmax >> 21);
    __syncthreads();
    if (tid == 0) {
        int top = 0;
        for (int w = 0; w < kSampleThreads / 32; ++w)
            top = max(top, warp_sums[w]);
        sh_lo = nloc > 0 && top >= 4 ? top - 4 : 0;
    }
    __syncthreads();
    unsigned* const rhist = cluster.map_shared_rank(hist, 0);
    cluster_wait();  // rank 0's histograms are zeroed
    unsigned prefix = 0u;
    int remaining = k;
    bool gather_all = false;
#pragma unroll 1
    for (int p = 0; p < 4; ++p) {  // p = 1 is the full pass 0, run only when needed
        const int digit_pass = p < 2 ? 0 : p - 1;
        const int shift = digit_pass == 0 ? 21 : (digit_pass == 1 ? 10 : 0);
        const int width = digit_pass == 2 ? 10 : 11;
        const unsigned high_mask = digit_pass == 0 ? 0u : (0xFFFFFFFFu << (shift + width));
        const unsigned dmask = (1u << width) - 1u;
        const int lo = p == 0 ? sh_lo : 0;
        unsigned* rh = rhist + p * kHistBins;
        for (int b = tid; b < kHistBins; b += kSampleThreads)
            hloc[b] = 0u;
        __syncthreads();
        for (int j = tid; j < nloc; j += kSampleThreads) {
            const unsigned key = keys_loc[j];
            if ((key & high_mask) == prefix) {
                const unsigned d = (key >> shift) & dmask;
                if ((int)d >= lo)
                    warp_count(hloc, d, lane);
            }
        }
        __syncthreads();
        for (int b = tid; b < kHistBins; b += kSampleThreads)  // one remote add per nonzero bin
            if (hloc[b] != 0u)
                atomicAdd(&rh[b], hloc[b]);
        cluster.sync();
        if (p == 0 && warp == 0) {  // the largest pass-0 bound of the cluster
            int l = lane < C ? *cluster.map_shared_rank(&sh_lo, lane) : 0;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
                l = max(l, __shfl_xor_sync(0xffffffffu, l, o));
            if (lane == 0)
                sh_lo_max = l;
        }
        // thread t owns the digits nb-1-2t and nb-2-2t (descending order)
        const int nb = 1 << width, d0 = nb - 1 - 2 * tid, d1 = d0 - 1;
        int g0 = d0 >= 0 ? (int)rh[d0] : 0, g1 = d1 >= 0 ? (int)rh[d1] : 0;
        if (p == 0) {
            __syncthreads();
            const int lmax = sh_lo_max;
            g0 = d0 >= lmax ? g0 : 0;
            g1 = d1 >= lmax ? g1 : 0;
        }
        int above;
        const int counted = block_exclusive_scan(g0 + g1, above, warp_sums);
        if (p == 0) {
            if (counted >= remaining)
                ++p;  // exact: skip the full pass 0
            else
                continue;
        }
        if (d0 >= 0) {
            if (above < remaining && above + g0 >= remaining) {
                sh_prefix = prefix | ((unsigned)d0 << shift);
                sh_remaining = remaining - above;
                sh_digit_count = g0;
                sh_gathered = above + g0;
            } else if (d1 >= 0 && above + g0 < remaining && above + g0 + g1 >= remaining) {
                sh_prefix = prefix | ((unsigned)d1 << shift);
                sh_remaining = remaining - above - g0;
                sh_digit_count = g1;
                sh_gathered = above + g0 + g1;
            }
        }
        __syncthreads();
        prefix = sh_prefix;
        remaining = sh_remaining;
        if (p == 1 && sh_gathered <= a.cap) {
            gather_all = true;
            break;
        }
    }

    unsigned* rkeys = cluster.map_shared_rank(gkeys, 0);
    int* ridx = cluster.map_shared_rank(gidx, 0);
    int* slots = cluster.map_shared_rank(&sh_slots, 0);
    if (gather_all) {
        // every key whose pass-0 digit is the selected one or larger (prefix holds that digit): the
        // CTA counts its keys, reserves one range in rank 0, and fills it through a local counter
        int mine = 0;
        for (int j = tid; j < nloc; j += kSampleThreads)
            mine += keys_loc[j] >= prefix;
        mine = __reduce_add_sync(0xffffffffu, mine);
        if (lane == 0)
            warp_sums[warp] = mine;
        __syncthreads();
        if (tid == 0) {
            int t = 0;
            for (int w = 0; w < kSampleThreads / 32; ++w)
                t += warp_sums[w];
            sh_tot[0] = t > 0 ? atomicAdd(slots, t) : 0;  // this CTA's range in rank 0's buffer
            sh_tot[1] = 0;
        }
        __syncthreads();
        for (int j = tid; j < nloc; j += kSampleThreads) {
            const unsigned key = keys_loc[j];
            warp_append(key >= prefix, key, base + j, &sh_tot[1], rkeys + sh_tot[0], ridx + sh_tot[0], lane);
        }
    } else {
        const unsigned thr = prefix;
        const int need_eq = remaining;  // keys equal to thr to take, lowest indices first
        if (sh_digit_count == need_eq) {
            // every key >= thr is a candidate (sh_digit_count: the keys equal to thr)
            for (int j = tid; j < nloc; j += kSampleThreads) {
                const unsigned key = keys_loc[j];
                warp_append(key >= thr, key, base + j, slots, rkeys, ridx, lane);
            }
        } else {
            // ties straddle the cut: the lowest indices among keys == thr, so each thread scans a
            // contiguous range and the ranges are ranked by a block scan and by CTA rank
            const int per = (nloc + kSampleThreads - 1) / kSampleThreads;
            const int i0 = min(nloc, tid * per), i1 = min(nloc, i0 + per);
            int ngt = 0, neq = 0;
            for (int j = i0; j < i1; ++j) {
                const unsigned key = keys_loc[j];
                ngt += key > thr;
                neq += key == thr;
            }
            int excl;
            const int tot = block_exclusive_scan(ngt | (neq << 16), excl, warp_sums);  // each count < 2^16
            if (tid == 0)
                sh_tot[0] = tot & 0xFFFF, sh_tot[1] = tot >> 16;
            cluster.sync();
            if (tid == 0) {
                int gb = 0, eb = 0, ga = 0;
                for (int r = 0; r < C; ++r) {
                    const int* rt = cluster.map_shared_rank(&sh_tot[0], r);
                    const int g = rt[0], e = rt[1];
                    if (r < rank)
                        gb += g, eb += e;
                    ga += g;
                }
                sh_offs[0] = gb, sh_offs[1] = eb, sh_offs[2] = ga;
            }
            __syncthreads();
            int og = sh_offs[0] + (excl & 0xFFFF), oe = sh_offs[1] + (excl >> 16);
            const int gt_all = sh_offs[2];
            for (int j = i0; j < i1; ++j) {
                const unsigned key = keys_loc[j];
                if (key > thr) {
                    rkeys[og] = key;
                    ridx[og] = base + j;
                    ++og;
                } else if (key == thr) {
                    if (oe < need_eq) {
                        rkeys[gt_all + oe] = key;
                        ridx[gt_all + oe] = base + j;
                    }
                    ++oe;
                }
            }
            if (rank == 0 && tid == 0)
                sh_slots = k;  // no CTA reserves slots on this path
        }
    }
    cluster.sync();  // candidates visible in rank 0; no CTA reads another's shared memory after this
    if (rank != 0)
        return;

    // 5. rank 0: the m candidates ordered by (key descending, id ascending); the first k are the
    // top-k. Then the weights and the draw.
    const int m = sh_slots;
    const int Kp = sample_pow2(k);
    const int SK = min(Kp, kRankSortMax);
    unsigned* skeys = reinterpret_cast<unsigned*>(smem_raw + a.cand_off + 8 * a.cap);
    int* sidx = reinterpret_cast<int*>(skeys + SK);
    double* w = reinterpret_cast<double*>(smem_raw + a.cand_off + 8 * a.cap + 8 * SK);
    double* q = w + k;    // w / total
    double* pre = q + k;  // left-to-right prefix sums of w
    const unsigned* keys;
    const int* idx;
    if (m <= kRankSortMax) {  // rank by counting: thread j places candidate j
        if (tid < m) {
            const unsigned mk = gkeys[tid];
            const int mi = gidx[tid];
            int r = 0;
            for (int j = 0; j < m; ++j) {
                const unsigned kj = gkeys[j];
                const int ij = gidx[j];
                r += kj > mk || (kj == mk && ij < mi);
            }
            if (r < k)
                skeys[r] = mk, sidx[r] = mi;
        }
        keys = skeys;
        idx = sidx;
    } else {  // bitonic sort of the gather buffer in place, padded to a power of two (<= a.cap)
        const int P = max(sample_pow2(m), 256);
        for (int j = m + tid; j < P; j += kSampleThreads)  // padding sorts last
            gkeys[j] = 0u, gidx[j] = INT_MAX;
        __syncthreads();
        if (P <= kSampleThreads)
            bitonic_sort_regs<1>(gkeys, gidx, P);
        else if (P == 2 * kSampleThreads)
            bitonic_sort_regs<2>(gkeys, gidx, P);
        else if (P == 4 * kSampleThreads)
            bitonic_sort_regs<4>(gkeys, gidx, P);
        else
            bitonic_sort_regs<8>(gkeys, gidx, P);
        keys = gkeys;
        idx = gidx;
    }
    __syncthreads();
    // engine refill (every 312 draws) in three phases equal to the sequential recurrence:
    // i < 156 reads only old words; 156 <= i < 311 reads the new word i - 156; i = 311 reads the
    // new words 0 and 155.
    if (mt_idx >= 312) {
        unsigned long long nv = 0;
        if (tid < 156)
            nv = mt64_twist(mt[tid], mt[tid + 1], mt[tid + 156]);
        __syncthreads();
        if (tid < 156)
            mt[tid] = nv;
        __syncthreads();
        if (tid >= 156 && tid < 311)
            nv = mt64_twist(mt[tid], mt[tid + 1], mt[tid - 156]);
        __syncthreads();
        if (tid >= 156 && tid < 311)
            mt[tid] = nv;
        __syncthreads();
        if (tid == 0) {
            mt[311] = mt64_twist(mt[311], mt[0], mt[155]);
            mt_idx = 0;
        }
        __syncthreads();
        for (int j = tid; j < 312; j += kSampleThreads)
            a.rng->mt[j] = mt[j];
    }
    const float lmax = key_value(keys[0]);
    for (int j = tid; j < k; j += kSampleThreads)
        w[j] = exp((double)(key_value(keys[j]) - lmax));
    __syncthreads();
    if (tid == 0)
        sh_total = ordered_prefix(w, pre, k);  // the reference's total; pre[j] = its running sum
    __syncthreads();
    const double total = sh_total;
    for (int j = tid; j < k; j += kSampleThreads)
        q[j] = w[j] / total;
    __syncthreads();
    // the nucleus sum runs in order over q; the kept mass and the draw's running sum are prefixes
    // of the same left-to-right sum over w as the total, so they come from pre[]
    if (tid == 0) {
        const int cut = first_reaching(q, k, (double)a.top_p);
        const int kept = cut < k ? cut + 1 : k;
        const unsigned long long y = mt64_temper(mt[mt_idx]);
        a.rng->idx = mt_idx + 1;
        double u = __ull2double_rn(y) * 0x1p-64;
        if (u >= 1.0)
            u = nextafter(1.0, 0.0);
        sh_total = u * pre[kept - 1];  // the draw's target
        sh_remaining = kept;
    }
    __syncthreads();
    const double target = sh_total;
    const int kept = sh_remaining;
    for (int j = tid; j < kept; j += kSampleThreads)  // the first running sum that reaches the target
        if (pre[j] >= target && (j == 0 || !(pre[j - 1] >= target)))
            atomicMin(&sh_hit, j);
    __syncthreads();
    if (tid == 0) {
        const int hit = sh_hit;
        const int token = idx[hit < kept ? hit : kept - 1];
        *a.token = token;
        if (a.gate)
            a.tokens[n] = token;
    }
}

}  // namespace muyo

using namespace muyo;

extern "C" size_t muyo_sampler_state_bytes(void) { return sizeof(Mt64State); }

extern "C" int muyo_sampler_seed(void* state, uint64_t seed, void* stream)
{
    clear_error();
    MUYO_REQUIRE(state && (reinterpret_cast<uintptr_t>(state) & 7u) == 0, "sampler_seed: state must be 8-byte aligned");
    k_mt64_seed<<<1, 1, 0, as_stream(stream)>>>(static_cast<Mt64State*>(state), (unsigned long long)seed);
    MUYO_LAUNCH_CHECK();
    return MUYO_OK;
}

static int sample_k(const MuyoSamplerParams* p, uint32_t vocab)
{
    if (!(p->temperature > 0.0f))
        return 1;
    return (int)(p->top_k <= 0 ? vocab : ((uint32_t)p->top_k < vocab ? (uint32_t)p->top_k : vocab));
}

// Per device: 1 when a 16-CTA cluster (one CTA per SM) can be placed, -1 when it cannot, 0 not yet
// known. Found by sample_check outside any stream capture; a capture reuses the answer.
static int g_cluster16[64];

static int device_index()
{
    int d = 0;
    return cudaGetDevice(&d) == cudaSuccess && d >= 0 && d < 64 ? d : 0;
}

// Cluster size and slice for a vocabulary: 16 CTAs when the device places them (more SMs share the
// row), else 8; `force` (8 or 16) overrides. The slice must fit shared memory and 16-bit counts.
static int sample_shape(uint32_t vocab, int k, uint32_t force, int& cluster, int& slice, SampleSmem& sm)
{
    const bool c16 = g_cluster16[device_index()] > 0;
    const int order[2] = {force == 8 || (force == 0 && !c16) ? 8 : 16, force == 8 || (force == 0 && !c16) ? 16 : 8};
    for (int i = 0; i < (force ? 1 : 2); ++i) {
        const int c = order[i];
        slice = (int)(((vocab + (uint32_t)c - 1) / (uint32_t)c + 3) / 4 * 4);
        for (int cap : {8192, 4096}) {
            if (cap < sample_pow2(k))
                continue;
            sm = sample_smem(slice, k, cap);
            if (sm.bytes <= kSmemMax && slice < 65536) {
                cluster = c;
                return MUYO_OK;
            }
        }
    }
    set_error("sample: a vocabulary of %u does not fit the device sampler's cluster", vocab);
    return MUYO_EUNSUPPORTED;
}

static void sample_config(cudaLaunchConfig_t& cfg, cudaLaunchAttribute* attr, int cluster, const SampleSmem& sm,
                          bool pdl, cudaStream_t s)
{
    cfg = cudaLaunchConfig_t{};
    cfg.gridDim = dim3(cluster);
    cfg.blockDim = dim3(kSampleThreads);
    cfg.dynamicSmemBytes = (size_t)sm.bytes;
    cfg.stream = s;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
}

// Checks a parameter block against what the device sampler supports and that its cluster can be
// placed on the current device (MUYO_OK or an error code; not during a stream capture).
// max_hist: the longest history a call can see (the penalty's 16-bit occurrence counts).
int sample_check(const MuyoSamplerParams* p, uint32_t vocab, long long max_hist)
{
    MUYO_REQUIRE(p, "sample: null parameter block");
    MUYO_REQUIRE(vocab > 0 && vocab <= (uint32_t)INT_MAX, "sample: vocab must be positive");
    MUYO_REQUIRE(!(p->temperature > 0.0f) || p->repeat_penalty == p->repeat_penalty, "sample: repeat_penalty is NaN");
    const long long window = p->repeat_last_n >= 0 && p->repeat_last_n < max_hist ? p->repeat_last_n : max_hist;
    if (p->repeat_penalty != 1.0f && window > 65535) {
        set_error("sample: a penalty window of %lld ids exceeds the device sampler's 65535", window);
        return MUYO_EUNSUPPORTED;
    }
    const int k = sample_k(p, vocab);
    if (k > kSampleMaxK) {
        set_error("sample: top-k of %d candidates exceeds the device sampler's %d", k, kSampleMaxK);
        return MUYO_EUNSUPPORTED;
    }
    MUYO_REQUIRE(p->cluster_ctas == 0 || p->cluster_ctas == 8 || p->cluster_ctas == 16,
                 "sample: cluster_ctas must be 0, 8 or 16");
    // always the largest values: a recorded graph's launch keeps its own sizes
    MUYO_CUDA_TRY(cudaFuncSetAttribute(k_sample, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax));
    MUYO_CUDA_TRY(cudaFuncSetAttribute(k_sample, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[2];
    int& c16 = g_cluster16[device_index()];
    if (c16 == 0) {  // one CTA of the largest shared-memory size per SM, 16 SMs in one cluster
        sample_config(cfg, attr, 16, SampleSmem{0, 0, kSmemMax, 0}, false, nullptr);
        int clusters = 0;
        MUYO_CUDA_TRY(cudaOccupancyMaxActiveClusters(&clusters, k_sample, &cfg));
        c16 = clusters >= 1 ? 1 : -1;
    }
    int cluster = 0, slice = 0;
    SampleSmem sm;
    int rc = sample_shape(vocab, k, p->cluster_ctas, cluster, slice, sm);
    if (rc)
        return rc;
    sample_config(cfg, attr, cluster, sm, false, nullptr);
    int clusters = 0;
    MUYO_CUDA_TRY(cudaOccupancyMaxActiveClusters(&clusters, k_sample, &cfg));
    if (clusters < 1) {
        set_error("sample: a cluster of %d CTAs with %d bytes of shared memory each cannot be placed", cluster,
                  sm.bytes);
        return MUYO_EUNSUPPORTED;
    }
    return MUYO_OK;
}

// gate/tokens/max_seq: the decode-graph mode of k_sample (gate == nullptr for a plain call). In a
// stream capture the parameters must have passed sample_check before (the model's set_sampler).
// pdl = false in the decode graph: launched early, the cluster would hold SM slots that the LM
// head's single-wave grid counts on.
int sample_launch(const MuyoSamplerParams* p, float* logits, uint32_t vocab, const int32_t* history,
                  uint32_t hist_len, void* state, int32_t* token, const int32_t* gate, int32_t* tokens,
                  int max_seq, bool pdl, cudaStream_t s)
{
    MUYO_REQUIRE(p && logits && state && token, "sample: null parameter block or buffer");
    MUYO_REQUIRE((reinterpret_cast<uintptr_t>(state) & 7u) == 0, "sample: state must be 8-byte aligned");
    MUYO_REQUIRE(hist_len == 0 || history, "sample: history is null");
    MUYO_REQUIRE(!gate || tokens, "sample: gated call without a token buffer");
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    MUYO_CUDA_TRY(cudaStreamIsCapturing(s, &cap));
    int rc = MUYO_OK;
    if (cap == cudaStreamCaptureStatusNone) {
        rc = sample_check(p, vocab, gate ? (long long)max_seq : (long long)hist_len);
        if (rc)
            return rc;
    }
    const int k = sample_k(p, vocab);
    int cluster = 0, slice = 0;
    SampleSmem sm;
    rc = sample_shape(vocab, k, p->cluster_ctas, cluster, slice, sm);
    if (rc)
        return rc;
    SampleArgs a{};
    a.temperature = p->temperature, a.top_k = p->top_k, a.top_p = p->top_p, a.repeat_penalty = p->repeat_penalty;
    a.repeat_last_n = p->repeat_last_n, a.vocab = (int)vocab, a.logits = logits, a.history = history;
    a.hist_len = (int)hist_len, a.rng = static_cast<Mt64State*>(state), a.token = token;
    a.gate = gate, a.tokens = tokens, a.max_seq = max_seq;
    a.slice = slice, a.cand_off = sm.cand_off, a.hist_off = sm.hist_off, a.cap = sm.cap;
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[2];
    sample_config(cfg, attr, cluster, sm, pdl, s);
    MUYO_CUDA_TRY(cudaLaunchKernelEx(&cfg, k_sample, a));
    MUYO_LAUNCH_CHECK();
    return MUYO_OK;
}

extern "C" int muyo_cuda_sample(const MuyoSamplerParams* p, float* logits, uint32_t vocab, const int32_t* history,
                                uint32_t hist_len, void* state, int32_t* token, void* stream)
{
    clear_error();
    return sample_launch(p, logits, vocab, history, hist_len, state, token, nullptr, nullptr, 0, true,
                         as_stream(stream));
}
