// On-device token sampler: Sampler::Sample (src/Sampler.cpp:10-98) with its std::mt19937_64 stream
// kept in device memory, so that non-greedy decoding needs no host round trip.
//
// One CTA of 1024 threads, in the reference's order:
//   1. repetition penalty over the history window, applied by one thread in history order (a token
//      that repeats is penalised once per occurrence, as in the reference);
//   2. temperature <= 0: the first index of the maximum (block argmax);
//   3. logits /= temperature, in place;
//   4. top-k: a 4-pass MSB-first radix select finds the k-th largest value; the candidates (ties at
//      the threshold by lower index, each thread owning a contiguous index range) are sorted by
//      (logit descending, index ascending) with a bitonic sort in shared memory;
//   5. weights exp(double(l_i - l_0)) in parallel; one thread then forms the sums in order (double),
//      the nucleus cut, draws u = canonical double from the engine and picks the token.
// mt19937_64 is restated from its published definition (Matsumoto & Nishimura): n = 312, m = 156,
// r = 31, a = 0xB5026F5AA96619E9, tempering (29, 0x5555555555555555), (17, 0x71D67FFFEDA60000),
// (37, 0xFFF7EEE000000000), 43; seeding multiplier 6364136223846793005.
#include <climits>
#include <cmath>

#include "common.cuh"

namespace muyo {

constexpr int kSampleThreads = 1024;
constexpr int kSampleMaxK = 4096;

struct Mt64State {
    unsigned long long mt[312];
    int idx;
    int pad;
};

__device__ unsigned long long mt64_next(Mt64State* s)
{
    const unsigned long long upper = 0xFFFFFFFF80000000ULL, lower = 0x7FFFFFFFULL, a = 0xB5026F5AA96619E9ULL;
    if (s->idx >= 312) {
        for (int i = 0; i < 312; ++i) {
            const unsigned long long x = (s->mt[i] & upper) | (s->mt[(i + 1) % 312] & lower);
            unsigned long long xa = x >> 1;
            if (x & 1ULL)
                xa ^= a;
            s->mt[i] = s->mt[(i + 156) % 312] ^ xa;
        }
        s->idx = 0;
    }
    unsigned long long y = s->mt[s->idx++];
    y ^= (y >> 29) & 0x5555555555555555ULL;
    y ^= (y << 17) & 0x71D67FFFEDA60000ULL;
    y ^= (y << 37) & 0xFFF7EEE000000000ULL;
    y ^= y >> 43;
    return y;
}

__global__ void k_mt64_seed(Mt64State* s, unsigned long long seed)
{
    s->mt[0] = seed;
    for (int i = 1; i < 312; ++i)
        s->mt[i] = 6364136223846793005ULL * (s->mt[i - 1] ^ (s->mt[i - 1] >> 62)) + (unsigned long long)i;
    s->idx = 312;
}

// Order-preserving unsigned key of a float (ascending); -0 is folded onto +0, which compares equal.
__device__ __forceinline__ unsigned sort_key(float f)
{
    unsigned b = __float_as_uint(f);
    if (b == 0x80000000u)
        b = 0u;
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
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
};

__global__ void __launch_bounds__(kSampleThreads) k_sample(SampleArgs a)
{
    extern __shared__ unsigned char smem_raw[];
    unsigned* keys = reinterpret_cast<unsigned*>(smem_raw);                        // [kSampleMaxK]
    int* idx = reinterpret_cast<int*>(smem_raw + sizeof(unsigned) * kSampleMaxK);  // [kSampleMaxK]
    double* w = reinterpret_cast<double*>(smem_raw + 8 * kSampleMaxK);           // [kSampleMaxK]
    __shared__ unsigned hist[256];
    __shared__ int warp_sums[32];
    __shared__ unsigned sh_prefix;
    __shared__ int sh_remaining, sh_token;
    __shared__ float sv[32];
    __shared__ int si[32];
    pdl_wait();
    pdl_trigger();
    const int tid = threadIdx.x, V = a.vocab;
    float* lg = a.logits;
    int hist_len = a.hist_len;
    const int32_t* history = a.history;
    int n = 0;
    if (a.gate) {  // uniform over the block: every thread reads the same words
        n = __ldcg(a.gate);
        if (n < __ldcg(a.gate + 1) || n >= __ldcg(a.gate + 2) || n >= a.max_seq)
            return;
        hist_len = n;
        history = a.tokens;
    }

    // 1. repetition penalty, in history order
    if (tid == 0 && a.repeat_penalty != 1.0f && hist_len > 0) {
        int begin = 0;
        if (a.repeat_last_n >= 0 && a.repeat_last_n < hist_len)
            begin = hist_len - a.repeat_last_n;
        for (int i = begin; i < hist_len; ++i) {
            const int t = history[i];
            if (t < 0 || t >= V)
                continue;
            const float v = lg[t];
            lg[t] = v > 0.0f ? __fdiv_rn(v, a.repeat_penalty) : v * a.repeat_penalty;
        }
    }
    __syncthreads();

    if (a.temperature <= 0.0f) {  // 2. greedy: the first index of the maximum
        float bv = -INFINITY;
        int bi = INT_MAX;
        for (int i = tid; i < V; i += blockDim.x)
            if (pair_better(lg[i], i, bv, bi))
                bv = lg[i], bi = i;
        warp_argmax(bv, bi);
        if ((tid & 31) == 0)
            sv[tid >> 5] = bv, si[tid >> 5] = bi;
        __syncthreads();
        if (tid < 32) {
            bv = sv[tid], bi = si[tid];
            warp_argmax(bv, bi);
            if (tid == 0)
                sh_token = bi == INT_MAX ? 0 : bi;
        }
        __syncthreads();
    } else {
        // 3. temperature, in place
        for (int i = tid; i < V; i += blockDim.x)
            lg[i] = __fdiv_rn(lg[i], a.temperature);
        __syncthreads();
        const int k = a.top_k <= 0 ? V : min(a.top_k, V);
        // 4. radix select of the k-th largest key, 8 bits per pass from the top
        if (tid == 0) {
            sh_prefix = 0u;
            sh_remaining = k;
        }
        for (int shift = 24; shift >= 0; shift -= 8) {
            for (int b = tid; b < 256; b += blockDim.x)
                hist[b] = 0u;
            __syncthreads();
            const unsigned prefix = sh_prefix;
            const unsigned high_mask = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
            for (int i = tid; i < V; i += blockDim.x) {
                const unsigned key = sort_key(lg[i]);
                if ((key & high_mask) == prefix)
                    atomicAdd(&hist[(key >> shift) & 0xFFu], 1u);
            }
            __syncthreads();
            if (tid == 0) {
                int remaining = sh_remaining;
                int b = 255;
                for (; b > 0; --b) {
                    if ((int)hist[b] >= remaining)
                        break;
                    remaining -= (int)hist[b];
                }
                sh_prefix = prefix | ((unsigned)b << shift);
                sh_remaining = remaining;  // elements still needed from the keys equal to the prefix so far
            }
            __syncthreads();
        }
        const unsigned thr = sh_prefix;
        const int need_eq = sh_remaining;  // how many keys == thr to take (lowest indices first)
        // gather: each thread scans a contiguous index range, so ties are ranked by index
        const int per = (V + blockDim.x - 1) / blockDim.x, i0 = min(V, tid * per), i1 = min(V, i0 + per);
        int n_gt = 0, n_eq = 0;
        for (int i = i0; i < i1; ++i) {
            const unsigned key = sort_key(lg[i]);
            n_gt += key > thr;
            n_eq += key == thr;
        }
        int off_gt = 0, off_eq = 0;
        const int total_gt = block_exclusive_scan(n_gt, off_gt, warp_sums);
        block_exclusive_scan(n_eq, off_eq, warp_sums);
        for (int i = i0; i < i1; ++i) {
            const unsigned key = sort_key(lg[i]);
            if (key > thr) {
                keys[off_gt] = key;
                idx[off_gt] = i;
                ++off_gt;
            } else if (key == thr) {
                if (off_eq < need_eq) {
                    keys[total_gt + off_eq] = key;
                    idx[total_gt + off_eq] = i;
                }
                ++off_eq;
            }
        }
        // pad to a power of two with entries that sort last
        int P = 1;
        while (P < k)
            P <<= 1;
        for (int j = k + tid; j < P; j += blockDim.x) {
            keys[j] = 0u;
            idx[j] = INT_MAX;
        }
        __syncthreads();
        // bitonic sort: (key descending, index ascending)
        for (int size = 2; size <= P; size <<= 1) {
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                for (int j = tid; j < P; j += blockDim.x) {
                    const int partner = j ^ stride;
                    if (partner > j) {
                        const bool desc_block = (j & size) == 0;  // this half of the merge is in final order
                        const unsigned ka = keys[j], kb = keys[partner];
                        const int ia = idx[j], ib = idx[partner];
                        const bool a_first = ka > kb || (ka == kb && ia < ib);
                        if (a_first != desc_block) {
                            keys[j] = kb, keys[partner] = ka;
                            idx[j] = ib, idx[partner] = ia;
                        }
                    }
                }
                __syncthreads();
            }
        }
        // 5. weights in parallel, the sums and the draw in order by one thread
        const float lmax = lg[idx[0]];
        for (int j = tid; j < k; j += blockDim.x)
            w[j] = exp((double)(lg[idx[j]] - lmax));
        __syncthreads();
        if (tid == 0) {
            double total = 0.0;
            for (int j = 0; j < k; ++j)
                total += w[j];
            int kept = k;
            double cumulative = 0.0;
            for (int j = 0; j < k; ++j) {
                cumulative += w[j] / total;
                if (cumulative >= (double)a.top_p) {
                    kept = j + 1;
                    break;
                }
            }
            double kept_total = 0.0;
            for (int j = 0; j < kept; ++j)
                kept_total += w[j];
            double u = __ull2double_rn(mt64_next(a.rng)) * 0x1p-64;
            if (u >= 1.0)
                u = nextafter(1.0, 0.0);
            const double target = u * kept_total;
            double acc = 0.0;
            int token = idx[kept - 1];
            for (int j = 0; j < kept; ++j) {
                acc += w[j];
                if (acc >= target) {
                    token = idx[j];
                    break;
                }
            }
            sh_token = token;
        }
        __syncthreads();
    }
    if (tid == 0) {
        *a.token = sh_token;
        if (a.gate)
            a.tokens[n] = sh_token;
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

// Checks a parameter block against what the device sampler supports (MUYO_OK or an error code).
int sample_check(const MuyoSamplerParams* p, uint32_t vocab)
{
    MUYO_REQUIRE(p, "sample: null parameter block");
    MUYO_REQUIRE(vocab > 0 && vocab <= (uint32_t)INT_MAX, "sample: vocab must be positive");
    MUYO_REQUIRE(!(p->temperature > 0.0f) || p->repeat_penalty == p->repeat_penalty, "sample: repeat_penalty is NaN");
    if (p->temperature > 0.0f) {
        const uint32_t k = p->top_k <= 0 ? vocab : ((uint32_t)p->top_k < vocab ? (uint32_t)p->top_k : vocab);
        if (k > (uint32_t)kSampleMaxK) {
            set_error("sample: top-k of %u candidates exceeds the device sampler's %d", k, kSampleMaxK);
            return MUYO_EUNSUPPORTED;
        }
    }
    return MUYO_OK;
}

// gate/tokens/max_seq: the decode-graph mode of k_sample (gate == nullptr for a plain call).
// pdl = false in the decode graph: launched early, the 1024-thread CTA would hold an SM slot that
// the LM head's single-wave grid counts on.
int sample_launch(const MuyoSamplerParams* p, float* logits, uint32_t vocab, const int32_t* history,
                  uint32_t hist_len, void* state, int32_t* token, const int32_t* gate, int32_t* tokens,
                  int max_seq, bool pdl, cudaStream_t s)
{
    MUYO_REQUIRE(p && logits && state && token, "sample: null parameter block or buffer");
    MUYO_REQUIRE((reinterpret_cast<uintptr_t>(state) & 7u) == 0, "sample: state must be 8-byte aligned");
    MUYO_REQUIRE(hist_len == 0 || history, "sample: history is null");
    MUYO_REQUIRE(!gate || tokens, "sample: gated call without a token buffer");
    const int rc = sample_check(p, vocab);
    if (rc)
        return rc;
    SampleArgs a{};
    a.temperature = p->temperature, a.top_k = p->top_k, a.top_p = p->top_p, a.repeat_penalty = p->repeat_penalty;
    a.repeat_last_n = p->repeat_last_n, a.vocab = (int)vocab, a.logits = logits, a.history = history;
    a.hist_len = (int)hist_len, a.rng = static_cast<Mt64State*>(state), a.token = token;
    a.gate = gate, a.tokens = tokens, a.max_seq = max_seq;
    const size_t smem = 16 * (size_t)kSampleMaxK;  // keys + indices + weights
    MUYO_CUDA_TRY(cudaFuncSetAttribute(k_sample, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    MUYO_CUDA_TRY(launch_kernel(k_sample, dim3(1), dim3(kSampleThreads), smem, s, pdl, a));
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
