// Sampling beyond argmax: temperature, top-k and top-p over a logits row.
// The reference's predict is greedy only and leaves sampling as a TODO
// (cuda.cu:988); this is the extension its Generate loop would call instead of
// argmax (llm/model.go:116-178).
//
// Per row (one CTA of 1024 threads), deterministic for a given seed and step:
//   1. candidates: the K = min(top_k, 256) largest logits (top_k <= 0: 256),
//      ordered by value, equal values by smaller index -- found by a radix
//      select on the order-preserving bit pattern of each value (four 8-bit
//      passes over the row) and a bitonic sort of the K candidates;
//   2. e_i = exp((l_i - l_max) / temperature) in fp32, prefix sums c_i;
//   3. top-p: the shortest prefix whose sum reaches top_p * c_K (top_p <= 0 or
//      >= 1: all K);
//   4. u = uniform(seed, step, row) in [0, 1): the token is the first candidate
//      i of the prefix with c_i > u * c_m.
// uniform(): the top 24 bits of a 64-bit counter hash, times 2^-24.
#include "common.cuh"
#include "wukong_ext.h"
#include "wukong_internal.cuh"

namespace wk {

namespace {

constexpr int kSampleMaxK = 256;
constexpr int kSampleThreads = 1024;

__device__ __forceinline__ uint32_t order_key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ uint64_t mix64s(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

template <typename T>
__global__ void __launch_bounds__(kSampleThreads) sample_kernel(int *__restrict__ tokens, const T *__restrict__ logits,
                                                                long ld, int V, SampleArgs p) {
    __shared__ int hist[256];
    __shared__ uint32_t s_prefix;
    __shared__ int s_remaining, s_ng, s_eq_base[kSampleThreads / 32];
    __shared__ float cv[kSampleMaxK];
    __shared__ int ci[kSampleMaxK];
    const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const T *x = logits + (long)b * ld;
    const int K = min(p.top_k > 0 && p.top_k < kSampleMaxK ? p.top_k : kSampleMaxK, V);
    // blocked ranges so that a scan over threads follows the index order
    const int per = (V + kSampleThreads - 1) / kSampleThreads;
    const int lo = min(V, tid * per), hi = min(V, lo + per);
    pdl_wait();
    pdl_trigger();
    // ---- radix select of the K-th largest key
    uint32_t prefix = 0, mask = 0;
    if (tid == 0) s_remaining = K;
    for (int shift = 24; shift >= 0; shift -= 8) {
        if (tid < 256) hist[tid] = 0;
        __syncthreads();
        for (int i = lo; i < hi; ++i) {
            const uint32_t k = order_key(to_float(x[i]));
            if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 255], 1);
        }
        __syncthreads();
        if (tid == 0) {
            int rem = s_remaining, cum = 0, sel = 0;
            for (int bin = 255; bin >= 0; --bin) {
                if (cum + hist[bin] >= rem) {
                    sel = bin;
                    rem -= cum;
                    break;
                }
                cum += hist[bin];
            }
            s_remaining = rem;
            s_prefix = prefix | ((uint32_t)sel << shift);
        }
        __syncthreads();
        prefix = s_prefix;
        mask |= 255u << shift;
    }
    const uint32_t thr = prefix;         // key of the K-th largest value
    const int need_eq = s_remaining;     // values equal to it that are taken (smallest indices first)
    // ---- collect: every key above thr, and the first need_eq keys equal to it
    int ne = 0;
    for (int i = lo; i < hi; ++i) ne += order_key(to_float(x[i])) == thr;
    // exclusive scan of ne over threads (index order)
    int incl = ne;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) s_eq_base[wid] = incl;
    if (tid == 0) s_ng = 0;
    __syncthreads();
    if (tid == 0) {
        int run = 0;
        for (int w = 0; w < kSampleThreads / 32; ++w) {
            const int c = s_eq_base[w];
            s_eq_base[w] = run;
            run += c;
        }
    }
    if (tid < kSampleMaxK) {
        cv[tid] = -INFINITY;
        ci[tid] = 0x7fffffff;
    }
    __syncthreads();
    int eq_rank = s_eq_base[wid] + incl - ne;
    const int n_gt = K - need_eq;  // keys strictly above thr
    for (int i = lo; i < hi; ++i) {
        const float v = to_float(x[i]);
        const uint32_t k = order_key(v);
        int slot = -1;
        if (k > thr) {
            slot = atomicAdd(&s_ng, 1);
        } else if (k == thr) {
            if (eq_rank < need_eq) slot = n_gt + eq_rank;
            ++eq_rank;
        }
        if (slot >= 0 && slot < kSampleMaxK) {
            cv[slot] = v;
            ci[slot] = i;
        }
    }
    __syncthreads();
    // ---- bitonic sort of the 256 slots: value descending, index ascending
    for (int size = 2; size <= kSampleMaxK; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (tid < kSampleMaxK) {
                const int j = tid ^ stride;
                if (j > tid) {
                    const bool desc = (tid & size) == 0;
                    const float a = cv[tid], c = cv[j];
                    const int ia = ci[tid], ic = ci[j];
                    const bool a_first = a > c || (a == c && ia < ic);
                    if (a_first != desc) {
                        cv[tid] = c;
                        cv[j] = a;
                        ci[tid] = ic;
                        ci[j] = ia;
                    }
                }
            }
            __syncthreads();
        }
    }
    // ---- softmax over the candidates, top-p prefix, the draw (warp 0, 8 candidates per lane)
    if (wid == 0) {
        const float lmax = cv[0];
        const float invt = 1.0f / p.temperature;
        float e[8], c[8], run = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = lane * 8 + j;
            e[j] = i < K ? expf((cv[i] - lmax) * invt) : 0.f;
            run += e[j];
            c[j] = run;
        }
        // inclusive prefix sums across lanes
        float base = run;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float v = __shfl_up_sync(0xffffffffu, base, o);
            if (lane >= o) base += v;
        }
        const float off = base - run;
#pragma unroll
        for (int j = 0; j < 8; ++j) c[j] += off;
        const float total = __shfl_sync(0xffffffffu, base, 31);
        // shortest prefix reaching top_p of the total
        int m = K;
        if (p.top_p > 0.f && p.top_p < 1.f) {
            const float target = p.top_p * total;
            int first = K;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = lane * 8 + j;
                if (i < K && c[j] >= target) first = min(first, i);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) first = min(first, __shfl_xor_sync(0xffffffffu, first, o));
            m = first + 1;
        }
        const float cm = __shfl_sync(0xffffffffu, c[(m - 1) & 7], (m - 1) >> 3);
        const long long step = p.pos ? (long long)p.pos[(long)b * p.pos_stride + p.pos_off] : p.step;
        const uint64_t h = mix64s(p.seed + 0x9E3779B97F4A7C15ull * (uint64_t)(step * 65536 + b + 1));
        const float u = (float)(h >> 40) * (1.0f / 16777216.0f) * cm;
        int pick = m - 1;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = lane * 8 + j;
            if (i < m && c[j] > u) pick = min(pick, i);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) pick = min(pick, __shfl_xor_sync(0xffffffffu, pick, o));
        if (lane == 0) tokens[b] = ci[pick];
    }
}

}  // namespace

void sample_rows(int *tokens, const void *logits, long ld, int rows, int V, int act, const SampleArgs &p,
                 cudaStream_t s) {
    if (rows <= 0) return;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(rows);
    cfg.blockDim = dim3(kSampleThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = g_rt.pdl ? 1 : 0;
    if (act == kBF16)
        WK_CHECK(cudaLaunchKernelEx(&cfg, sample_kernel<__nv_bfloat16>, tokens, (const __nv_bfloat16 *)logits, ld, V, p));
    else if (act == kF32)
        WK_CHECK(cudaLaunchKernelEx(&cfg, sample_kernel<float>, tokens, (const float *)logits, ld, V, p));
    else
        WK_CHECK(cudaLaunchKernelEx(&cfg, sample_kernel<__half>, tokens, (const __half *)logits, ld, V, p));
}

}  // namespace wk

using namespace wk;

extern "C" {

int wk_sample_logits(int *tokens, const void *logits, int rows, int vocab, int dtype, float temperature, int top_k,
                     float top_p, unsigned long long seed, long long step) {
    if (g_rt.device < 0) return fail("wk_sample_logits: cuda_init() has not been called");
    if (rows < 1 || vocab < 1 || !tokens || !logits) return fail("wk_sample_logits: bad arguments");
    if (dtype != kF16 && dtype != kBF16 && dtype != kF32) return fail("wk_sample_logits: dtype %d", dtype);
    if (!(temperature > 0.f)) return fail("wk_sample_logits: temperature must be positive");
    set_device_current();
    SampleArgs p;
    p.temperature = temperature;
    p.top_k = top_k;
    p.top_p = top_p;
    p.seed = seed;
    p.step = step;
    sample_rows(tokens, logits, vocab, rows, vocab, dtype, p, stream());
    return 0;
}

}  // extern "C"
