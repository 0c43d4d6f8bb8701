// Causal GQA attention over a KV source (paged cache or contiguous QKV rows).
//
// Reference semantics (cuda.cu:767-852 with the scaled softmax of :673-765 and
// the K/V replication of :437-467), per query row i at position p:
//   s_j = T(q . k_j)                     (cuBLAS GEMM output stored as T)
//   e_j = exp(s_j * scale - max)         (fp32, scale = 1/sqrt(HS))
//   sum = sum_j e_j                      (fp32, of the unrounded e_j)
//   P_j = T(T(e_j) * (1 / sum))          (numerator stored as T, then rescaled)
//   o   = T(sum_j P_j v_j)               (fp32 accumulation)
// for keys j <= p.  This kernel computes exactly these rounding points in one
// pass per (query row, KV head): the GQA group's query heads share the K/V
// rows, which are read once per CTA (no replication, no permutes).
#include "common.cuh"
#include "wukong_internal.cuh"

namespace wk {

namespace {

struct KVPaged {
    const void *k, *v;
    const int *block_table;
    int max_pages, page, kv_heads, hd;
    __device__ __forceinline__ long off(int seq, int j, int kvh) const {
        const long pg = block_table[(long)seq * max_pages + j / page];
        return ((pg * kv_heads + kvh) * page + j % page) * hd;
    }
};

struct KVRows {
    const void *k, *v;   // base of K and V columns of row 0
    long seq_stride;     // elements between sequences
    long row_stride;     // elements between rows
    int hd;
    __device__ __forceinline__ long off(int seq, int j, int kvh) const {
        return (long)seq * seq_stride + (long)j * row_stride + (long)kvh * hd;
    }
};

template <typename T, typename KV>
__global__ void __launch_bounds__(128) attn_rows_kernel(T *__restrict__ out, long out_row_stride,
                                                        const T *__restrict__ q, long q_row_stride,
                                                        const int *__restrict__ seq_of_row,
                                                        const int *__restrict__ pos_of_row, int rows_per_seq, KV kv,
                                                        int H, int Hk, int D, float scale) {
    extern __shared__ __align__(16) float sh[];
    pdl_wait();
    pdl_trigger();
    const int kvh = blockIdx.x, row = blockIdx.y;
    const int G = H / Hk;
    // without per-row metadata, row = seq * rows_per_seq + position
    const int seq = seq_of_row ? seq_of_row[row] : row / rows_per_seq;
    const int pos = pos_of_row ? pos_of_row[row] : row % rows_per_seq;
    const int L = pos + 1;
    float *qs = sh;                    // [G][D]
    float *s = sh + G * D;             // [G][L]
    float *red = s + (long)G * L;      // [G][4] + [G] (two reductions)
    const T *qrow = q + (long)row * q_row_stride + (long)kvh * G * D;
    for (int i = threadIdx.x; i < G * D; i += blockDim.x) qs[i] = to_float(qrow[i]);
    __syncthreads();

    const T *K = reinterpret_cast<const T *>(kv.k);
    const T *V = reinterpret_cast<const T *>(kv.v);
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;

    // scores: one thread per key, all heads of the group
    float lmax[8];
#pragma unroll
    for (int g = 0; g < 8; ++g) lmax[g] = -INFINITY;
    for (int j = tid; j < L; j += blockDim.x) {
        const T *kr = K + kv.off(seq, j, kvh);
        float acc[8];
#pragma unroll
        for (int g = 0; g < 8; ++g) acc[g] = 0.f;
        for (int d = 0; d < D; ++d) {
            const float kd = to_float(kr[d]);
#pragma unroll
            for (int g = 0; g < 8; ++g)
                if (g < G) acc[g] += qs[g * D + d] * kd;
        }
#pragma unroll
        for (int g = 0; g < 8; ++g)
            if (g < G) {
                const float sv = round_to<T>(acc[g]);
                s[(long)g * L + j] = sv;
                lmax[g] = fmaxf(lmax[g], sv * scale);
            }
    }
    // block max per head
#pragma unroll
    for (int g = 0; g < 8; ++g)
        if (g < G) {
            float m = warp_max(lmax[g]);
            if (lane == 0) red[g * 4 + wid] = m;
        }
    __syncthreads();
    float gmax[8], gsum[8];
#pragma unroll
    for (int g = 0; g < 8; ++g)
        gmax[g] = g < G ? fmaxf(fmaxf(red[g * 4], red[g * 4 + 1]), fmaxf(red[g * 4 + 2], red[g * 4 + 3])) : 0.f;
    __syncthreads();
    // numerators (stored as T) and their fp32 sum
    float lsum[8];
#pragma unroll
    for (int g = 0; g < 8; ++g) lsum[g] = 0.f;
    for (int j = tid; j < L; j += blockDim.x) {
#pragma unroll
        for (int g = 0; g < 8; ++g)
            if (g < G) {
                const float e = expf(s[(long)g * L + j] * scale - gmax[g]);
                lsum[g] += e;
                s[(long)g * L + j] = round_to<T>(e);
            }
    }
#pragma unroll
    for (int g = 0; g < 8; ++g)
        if (g < G) {
            float v = warp_sum(lsum[g]);
            if (lane == 0) red[g * 4 + wid] = v;
        }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < 8; ++g) gsum[g] = g < G ? (red[g * 4] + red[g * 4 + 1]) + (red[g * 4 + 2] + red[g * 4 + 3]) : 1.f;
    for (int j = tid; j < L; j += blockDim.x) {
#pragma unroll
        for (int g = 0; g < 8; ++g)
            if (g < G) s[(long)g * L + j] = round_to<T>(s[(long)g * L + j] * (1.0f / gsum[g]));
    }
    __syncthreads();
    // o[g][d] = sum_j P[g][j] v_j[d]
    for (int i = tid; i < G * D; i += blockDim.x) {
        const int g = i / D, d = i % D;
        const float *p = s + (long)g * L;
        float acc = 0.f;
        for (int j = 0; j < L; ++j) acc += p[j] * to_float(V[kv.off(seq, j, kvh) + d]);
        out[(long)row * out_row_stride + (long)(kvh * G + g) * D + d] = from_float<T>(acc);
    }
}

template <typename T, typename KV>
void launch_rows(T *out, long out_rs, const T *q, long q_rs, const int *seq_of_row, const int *pos_of_row,
                 int rows_per_seq, int nrows, int max_len, const KV &kv, int H, int Hk, int D, cudaStream_t s,
                 bool pdl) {
    if (nrows <= 0) return;
    const int G = H / Hk;
    if (G > 8) WK_PANIC("attention: %d query heads per KV head (max 8)", G);
    size_t smem = sizeof(float) * ((size_t)G * D + (size_t)G * max_len + G * 4 + 8);
    if ((int)smem > g_rt.max_smem_optin)
        WK_PANIC("attention: context %d needs %zu B of shared memory", max_len, smem);
    auto kern = attn_rows_kernel<T, KV>;
    WK_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(Hk, nrows);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = (pdl && g_rt.pdl) ? 1 : 0;
    const float scale = 1.0f / sqrtf((float)D);
    WK_CHECK(cudaLaunchKernelEx(&cfg, kern, out, out_rs, q, q_rs, seq_of_row, pos_of_row, rows_per_seq, kv, H, Hk, D,
                                scale));
}

}  // namespace

template <typename T>
void attention_paged(T *out, long out_rs, const T *q, long q_rs, const int *seq_of_row, const int *pos_of_row,
                     int nrows, int max_len, const PagedKV &c, int H, cudaStream_t s, bool pdl) {
    KVPaged kv{c.k, c.v, c.block_table, c.max_pages, c.page, c.kv_heads, c.hd};
    launch_rows<T>(out, out_rs, q, q_rs, seq_of_row, pos_of_row, 1, nrows, max_len, kv, H, c.kv_heads, c.hd, s, pdl);
}
template void attention_paged<__half>(__half *, long, const __half *, long, const int *, const int *, int, int,
                                      const PagedKV &, int, cudaStream_t, bool);
template void attention_paged<__nv_bfloat16>(__nv_bfloat16 *, long, const __nv_bfloat16 *, long, const int *,
                                             const int *, int, int, const PagedKV &, int, cudaStream_t, bool);
template void attention_paged<float>(float *, long, const float *, long, const int *, const int *, int, int,
                                     const PagedKV &, int, cudaStream_t, bool);

// Causal attention straight from fused QKV rows [B, T, (NH + 2 kvNH) HS]
// (the layout cuda_gq_sdpa takes); out [B, T, NH HS].
template <typename T>
void attention_qkv_rows(T *out, const T *qkv, int B, int Tn, int NH, int kvNH, int HS, cudaStream_t s) {
    if (B <= 0 || Tn <= 0) return;
    const long W = (long)(NH + 2 * kvNH) * HS;
    KVRows kv{qkv + (long)NH * HS, qkv + (long)(NH + kvNH) * HS, (long)Tn * W, W, HS};
    launch_rows<T>(out, (long)NH * HS, qkv, W, nullptr, nullptr, Tn, B * Tn, Tn, kv, NH, kvNH, HS, s, false);
}
template void attention_qkv_rows<float>(float *, const float *, int, int, int, int, int, cudaStream_t);
template void attention_qkv_rows<__half>(__half *, const __half *, int, int, int, int, int, cudaStream_t);
template void attention_qkv_rows<__nv_bfloat16>(__nv_bfloat16 *, const __nv_bfloat16 *, int, int, int, int, int,
                                                cudaStream_t);

}  // namespace wk

using namespace wk;

extern "C" {

// cuda.cu:1182-1185: multi-head attention on [B, T, 3 * NH * HS] fp32 rows.
// Unlike the reference, the input buffer is left unmodified (the reference
// writes its P.V product into `inp`, cuda.cu:779).
void cuda_mh_sdpa(void *out, const void *inp, int batch, int row, int NH, int HS) {
    ensure_init();
    attention_qkv_rows<float>((float *)out, (const float *)inp, batch, row, NH, NH, HS, stream());
}

// cuda.cu:1139-1145
void cuda_gq_sdpa(void *out, const void *inp, int batch, int row, int qNH, int kvNH, int HS) {
    ensure_init();
    if (kvNH <= 0 || qNH % kvNH) WK_PANIC("qNH (%d) must be a multiple of kvNH (%d)", qNH, kvNH);
    attention_qkv_rows<float>((float *)out, (const float *)inp, batch, row, qNH, kvNH, HS, stream());
}

// cuda.cu:1197-1203
void cuda_mq_sdpa(void *out, const void *inp, int batch, int row, int qNH, int HS) {
    ensure_init();
    attention_qkv_rows<float>((float *)out, (const float *)inp, batch, row, qNH, 1, HS, stream());
}

}  // extern "C"
