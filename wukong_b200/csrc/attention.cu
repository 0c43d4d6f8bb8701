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
#include <stdlib.h>

#include "common.cuh"
#include "timeline.cuh"
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
    static int configured = 0;
    if ((int)smem > configured) {
        WK_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        configured = (int)smem;
    }
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

// ---------------------------------------------------------------------------
// Tensor-core variant for 16-bit paged caches (the decode path).
//
// One CTA (4 warps) per (query row, KV head); the G <= 8 query heads of the GQA
// group are the 8 columns of mma.sync m16n8k16 tiles:
//   S^T[16 keys x 8 heads] = K[16 keys x D] . Q^T[D x 8 heads]   (A by ldmatrix)
//   O^T[16 d x 8 heads]    = V^T[16 d x keys] . P^T[keys x 8]     (A by ldmatrix.trans)
// K and V pages ([page][kv_head][64 tokens][D], 8 or 16 KB contiguous per head)
// stream through a shared-memory ring of up to 64 KB by 1-D bulk copies; pages that
// precede the newest token's page were written by earlier launches and are
// requested before griddepcontrol.wait.  Between the two GEMM passes the
// softmax runs on the fp16 score row kept in shared memory with the
// reference's rounding points (see the file header).
constexpr int kAttnPage = 64;
constexpr int kAttnSlots = 4;     // ring slots of the split-K kernels
constexpr int kAttnMaxSlots = 8;  // of the decode kernel: up to 64 KB of pages, fewer for long contexts

template <typename T> struct IsBF16 {
    static constexpr bool value = false;
};
template <> struct IsBF16<__nv_bfloat16> {
    static constexpr bool value = true;
};

template <typename T>
__device__ __forceinline__ void mma16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                      uint32_t b1) {
    if constexpr (IsBF16<T>::value)
        mma_bf16(c, a0, a1, a2, a3, b0, b1);
    else
        mma_f16(c, a0, a1, a2, a3, b0, b1);
}

// Q of a GQA group into shared memory [8][D], zero-padded to 8 heads, with
// 16-byte loads (one round trip) when the row is 16-byte aligned
template <typename T, int D>
__device__ __forceinline__ void stage_q(T *qs, const T *qrow, int G) {
    const int tid = threadIdx.x;
    if ((reinterpret_cast<uintptr_t>(qrow) & 15) == 0) {
        const int nv = G * D / 8;
        for (int i = tid; i < D; i += 128)  // 8 heads x D / 8 uint4
            reinterpret_cast<uint4 *>(qs)[i] =
                i < nv ? reinterpret_cast<const uint4 *>(qrow)[i] : make_uint4(0u, 0u, 0u, 0u);
    } else {
        for (int i = tid; i < 8 * D; i += 128) qs[i] = i < G * D ? qrow[i] : from_float<T>(0.f);
    }
}

template <typename T, int D, int S>
__global__ void __launch_bounds__(128) attn_decode_tc_kernel(T *__restrict__ out, long out_rs, const T *__restrict__ q,
                                                             long q_rs, const int *__restrict__ seq_of_row,
                                                             const int *__restrict__ pos_of_row, KVPaged kv, int G,
                                                             int Lpad_max, float scale, int *err, const void *pf,
                                                             long pf_bytes, int early) {
    Timeline tl;
    constexpr int kPageBytes = kAttnPage * D * 2;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *ring = smem;                                                      // [slots][64][D] T
    uint64_t *bars = reinterpret_cast<uint64_t *>(ring + S * kPageBytes);   // S <= kAttnMaxSlots
    float *red = reinterpret_cast<float *>(bars + kAttnMaxSlots);             // [8 heads][4 warps]
    T *qs = reinterpret_cast<T *>(red + 64);                                  // [8][D]
    T *sc = qs + 8 * D;                                                       // [8][Lpad_max] scores -> P

    const int kvh = blockIdx.x, row = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int seq = seq_of_row[row], pos = pos_of_row[row];
    const int L = pos + 1;
    const int npages = (L + kAttnPage - 1) / kAttnPage;
    const int Lpad = npages * kAttnPage;
    const T *K = reinterpret_cast<const T *>(kv.k);
    const T *V = reinterpret_cast<const T *>(kv.v);
    // the sequence's page ids, read once (one round trip, not one per page copy)
    int *pgs = reinterpret_cast<int *>(sc + 8 * Lpad_max);
    const int *bt = kv.block_table + (long)seq * kv.max_pages;
    auto page_src = [&](int i) -> const T * {
        // units 0..npages-1 are K pages, npages..2*npages-1 the V pages
        const int p = i < npages ? i : i - npages;
        return (i < npages ? K : V) + ((long)pgs[p] * kv.kv_heads + kvh) * (long)kAttnPage * D;
    };
    if (tid == 64 && pf)
        l2_prefetch_slice(pf, pf_bytes, blockIdx.y * gridDim.x + blockIdx.x, gridDim.x * gridDim.y);
    if (tid < S) mbar_init(bars + tid, 1);
    // decode: the block table is not written by the producing kernel
    if (early)
        for (int i = tid; i < npages; i += 128) pgs[i] = bt[i];
    mbar_fence_init();
    __syncthreads();
    const int total = 2 * npages;
    // When every row is the newest token of its sequence (decode), the pages
    // before its page were written by earlier launches: fetch them before the
    // wait for the producing kernel.  Otherwise (several rows of a sequence in
    // this call) that kernel may still be writing them.
    int issued = 0;
    if (tid == 0 && early) {
        for (; issued < S && issued < npages - 1; ++issued) {
            mbar_expect_tx(bars + issued, kPageBytes);
            bulk_g2s(ring + issued * kPageBytes, page_src(issued), kPageBytes, bars + issued);
        }
        // the other complete pages (K past the ring, all V but the newest) go to L2
        for (int p = issued; p < npages - 1; ++p)
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(page_src(p)), "r"((uint32_t)kPageBytes)
                         : "memory");
        for (int p = 0; p < npages - 1; ++p)
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(page_src(npages + p)),
                         "r"((uint32_t)kPageBytes)
                         : "memory");
    }
    pdl_wait();
    pdl_trigger();
    tl.mark(100, npages, G);
    if (!early) {
        for (int i = tid; i < npages; i += 128) pgs[i] = bt[i];
        __syncthreads();
    }
    if (tid == 0) {
        for (; issued < S && issued < total; ++issued) {
            mbar_expect_tx(bars + issued, kPageBytes);
            bulk_g2s(ring + issued * kPageBytes, page_src(issued), kPageBytes, bars + issued);
        }
    }
    // Q of the group, zero-padded to 8 heads
    const T *qrow = q + (long)row * q_rs + (long)kvh * G * D;
    stage_q<T, D>(qs, qrow, G);
    __syncthreads();
    tl.phase(0);  // q staged
    uint32_t qb[D / 16][2];
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
        qb[kk][0] = *reinterpret_cast<const uint32_t *>(qs + g * D + kk * 16 + 2 * t);
        qb[kk][1] = *reinterpret_cast<const uint32_t *>(qs + g * D + kk * 16 + 2 * t + 8);
    }

    // ---- pass 1: scores, rounded to T, and the row max per head
    float mx0 = -INFINITY, mx1 = -INFINITY;  // heads 2t, 2t+1
    int consumed = 0;
    bool ok = true;
    for (int p = 0; p < npages; ++p, ++consumed) {
        const int slot = consumed % S;
        if (!mbar_wait_bounded(bars + slot, (consumed / S) & 1, err, 3)) ok = false;
        const T *kt = reinterpret_cast<const T *>(ring + slot * kPageBytes) + warp * 16 * D;
        float c[4] = {0.f, 0.f, 0.f, 0.f};
        if (ok) {
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
                uint32_t a0, a1, a2, a3;
                ldsm_x4(smem_u32(kt + (lane & 15) * D + kk * 16 + (lane >> 4) * 8), a0, a1, a2, a3);
                mma16<T>(c, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
            }
        }
        // c0, c1: key g, heads 2t, 2t+1; c2, c3: key g + 8
        const int k0 = p * kAttnPage + warp * 16 + g;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int key = k0 + (i >> 1) * 8, h = 2 * t + (i & 1);
            const float sv = key < L ? round_to<T>(c[i]) : -INFINITY;
            if (h < 8) sc[h * Lpad_max + key] = from_float<T>(key < L ? sv : 0.f);
            if (i & 1)
                mx1 = fmaxf(mx1, sv * scale);
            else
                mx0 = fmaxf(mx0, sv * scale);
        }
        __syncthreads();  // everyone is done with this slot
        if (tid == 0 && issued < total) {
            const int sl = issued % S;
            mbar_expect_tx(bars + sl, kPageBytes);
            bulk_g2s(ring + sl * kPageBytes, page_src(issued), kPageBytes, bars + sl);
            ++issued;
        }
    }
    tl.phase(1);  // scores
    // max over the 8 lanes sharing t (g = 0..7), then over warps
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
    }
    if (g == 0) {
        red[(2 * t) * 4 + warp] = mx0;
        red[(2 * t + 1) * 4 + warp] = mx1;
    }
    __syncthreads();
    // ---- softmax numerators: thread -> (head h, keys j = i, i + 16, ...)
    const int h = tid >> 4, i0 = tid & 15;  // 8 heads x 16 threads
    const float M = fmaxf(fmaxf(red[h * 4], red[h * 4 + 1]), fmaxf(red[h * 4 + 2], red[h * 4 + 3]));
    // keys j = i0 + 16 u; eight at a time so that the loads and exponentials
    // overlap, summed in ascending j as one at a time would
    T *srow = sc + h * Lpad_max;
    float lsum = 0.f;
    for (int j0 = i0; j0 < Lpad; j0 += 16 * 8) {
        float e[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int j = j0 + 16 * u;
            e[u] = j < L && h < G ? to_float(srow[j]) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int j = j0 + 16 * u;
            if (j < L && h < G) {
                e[u] = expf(e[u] * scale - M);
                lsum += e[u];
            }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (j0 + 16 * u < Lpad) srow[j0 + 16 * u] = from_float<T>(e[u]);
    }
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
    const float inv = 1.0f / lsum;
    if (h < G)
        for (int j0 = i0; j0 < L; j0 += 16 * 8) {
            float e[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (j0 + 16 * u < L) e[u] = to_float(srow[j0 + 16 * u]);
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (j0 + 16 * u < L) srow[j0 + 16 * u] = from_float<T>(e[u] * inv);
        }
    __syncthreads();

    tl.phase(2);  // softmax
    // ---- pass 2: O^T = V^T . P^T; warp w owns d-tiles w, w + 4
    constexpr int kDT = D / 16;
    float o[kDT > 4 ? 2 : 1][4];
#pragma unroll
    for (int a = 0; a < (kDT > 4 ? 2 : 1); ++a) o[a][0] = o[a][1] = o[a][2] = o[a][3] = 0.f;
    for (int p = 0; p < npages; ++p, ++consumed) {
        const int slot = consumed % S;
        if (!mbar_wait_bounded(bars + slot, (consumed / S) & 1, err, 3)) ok = false;
        if (p == npages - 1 && L % kAttnPage) {
            // rows past the sequence end hold stale cache bytes; their P is 0, but 0 * NaN is NaN
            T *vw = reinterpret_cast<T *>(ring + slot * kPageBytes);
            const int r0 = L - p * kAttnPage;
            for (int i = tid; i < (kAttnPage - r0) * D; i += 128) vw[r0 * D + i] = from_float<T>(0.f);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncthreads();
        }
        const T *vt = reinterpret_cast<const T *>(ring + slot * kPageBytes);
        if (ok) {
#pragma unroll
            for (int ks = 0; ks < kAttnPage / 16; ++ks) {
                const int key0 = p * kAttnPage + ks * 16;
                const uint32_t b0 = *reinterpret_cast<const uint32_t *>(sc + g * Lpad_max + key0 + 2 * t);
                const uint32_t b1 = *reinterpret_cast<const uint32_t *>(sc + g * Lpad_max + key0 + 2 * t + 8);
#pragma unroll
                for (int a = 0; a < (kDT > 4 ? 2 : 1); ++a) {
                    const int d0 = (warp + 4 * a) * 16;
                    if (d0 < D) {
                        const int mi = lane >> 3, r = lane & 7;
                        const T *addr = vt + (ks * 16 + r + (mi >> 1) * 8) * D + d0 + (mi & 1) * 8;
                        uint32_t a0, a1, a2, a3;
                        ldsm_x4_t(smem_u32(addr), a0, a1, a2, a3);
                        mma16<T>(o[a], a0, a1, a2, a3, b0, b1);
                    }
                }
            }
        }
        __syncthreads();
        if (tid == 0 && issued < total) {
            const int sl = issued % S;
            mbar_expect_tx(bars + sl, kPageBytes);
            bulk_g2s(ring + sl * kPageBytes, page_src(issued), kPageBytes, bars + sl);
            ++issued;
        }
    }
    tl.phase(3);  // P.V
    // o[a]: rows d0 + g, d0 + g + 8; columns (heads) 2t, 2t + 1
    T *orow = out + (long)row * out_rs + (long)kvh * G * D;
#pragma unroll
    for (int a = 0; a < (kDT > 4 ? 2 : 1); ++a) {
        const int d0 = (warp + 4 * a) * 16;
        if (d0 >= D) continue;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int d = d0 + g + (i >> 1) * 8, hh = 2 * t + (i & 1);
            if (hh < G) orow[(long)hh * D + d] = from_float<T>(o[a][i]);
        }
    }
}

// ---------------------------------------------------------------- decode attention over a CTA cluster
// One thread-block cluster of CS CTAs per (row, KV head); CTA z of the
// cluster takes the sequence's pages [z pps, (z + 1) pps).  The reference's
// rounding points need the row maximum before any exponential, so the CTAs
// exchange per-head values through distributed shared memory, separated by
// hardware cluster barriers:
//   1. s_j = T(q . k_j) for the own keys; the own maxima m_z (of s_j * scale)
//      go to every CTA of the cluster; M = max_z m_z;
//   2. e_j = exp(s_j * scale - M) stored as T in place; the own sums l_z of the
//      unrounded e_j go to every CTA; sum = l_0 + l_1 + ... in z order;
//   3. P_j = T(T(e_j) * (1 / sum)); the own partial o_z = P . V (fp32) goes to
//      the owner CTA of each output element (element e of the [G][D] group
//      output to CTA e % CS), which adds the CS partials in z order and stores
//      T(o).
// A cluster is scheduled as a unit and its CTAs wait only at the cluster
// barriers, so clusters may run in any number of waves.  Old pages (before the
// newest token's page) are requested before griddepcontrol.wait.
constexpr int kClusterMax = 16;  // CTAs per cluster (above 8 is a non-portable size)

struct ClusterSmem {
    size_t ring, bars, qs, sc, pgs, red, xm, xl, xo, total;
};
__host__ __device__ inline ClusterSmem cluster_smem(int D, int S, int pps, int CS) {
    ClusterSmem o;
    size_t p = 0;
    o.ring = p;
    p += (size_t)S * kAttnPage * D * 2;
    o.bars = p;
    p += 16 * 8;
    o.qs = p;
    p += (size_t)8 * D * 2;
    o.sc = p;
    p += (size_t)8 * pps * kAttnPage * 2;
    o.pgs = p;
    p += ((size_t)pps * 4 + 15) / 16 * 16;
    o.red = p;
    p += 8 * 4 * 4;
    o.xm = p;
    p += (size_t)CS * 8 * 4;
    o.xl = p;
    p += (size_t)CS * 8 * 4;
    o.xo = p;
    p += (size_t)CS * ((8 * D + CS - 1) / CS) * 4;
    o.total = p;
    return o;
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// store v at the same shared-memory offset as `local` in CTA `rank` of the cluster
__device__ __forceinline__ void st_cluster_f32(const float *local, uint32_t rank, float v) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(r), "f"(v) : "memory");
}

template <typename T, int D>
__global__ void __launch_bounds__(128) attn_cluster_kernel(T *__restrict__ out, long out_rs, const T *__restrict__ q,
                                                           long q_rs, const int *__restrict__ seq_of_row,
                                                           const int *__restrict__ pos_of_row, KVPaged kv, int G,
                                                           int CS, int pps, int S, float scale, int *err, int early) {
    Timeline tl;
    constexpr int kPageBytes = kAttnPage * D * 2;
    extern __shared__ __align__(128) uint8_t smem[];
    const ClusterSmem lay = cluster_smem(D, S, pps, CS);
    uint8_t *ring = smem + lay.ring;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + lay.bars);
    T *qs = reinterpret_cast<T *>(smem + lay.qs);
    T *sc = reinterpret_cast<T *>(smem + lay.sc);
    int *pgs = reinterpret_cast<int *>(smem + lay.pgs);
    float *red = reinterpret_cast<float *>(smem + lay.red);  // [8 heads][4 warps]
    float *xm = reinterpret_cast<float *>(smem + lay.xm);    // [CS][8] maxima of each CTA
    float *xl = reinterpret_cast<float *>(smem + lay.xl);    // [CS][8] exponent sums of each CTA
    float *xo = reinterpret_cast<float *>(smem + lay.xo);    // [CS][per] partial outputs of owned elements
    const int per = (8 * D + CS - 1) / CS;
    const int lpad = pps * kAttnPage;  // score row stride
    const int z = (int)cluster_ctarank();
    const int kvh = blockIdx.x / CS, row = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    // every CTA of the cluster has started before the first remote store (waited on below)
    cluster_arrive_relaxed();
    const int seq = seq_of_row[row], pos = pos_of_row[row];
    const int L = pos + 1;
    const int npages = (L + kAttnPage - 1) / kAttnPage;
    const int pbeg = z * pps;
    const int nloc = max(0, min(npages - pbeg, pps));  // own pages
    const int total = 2 * nloc;                        // units: own K pages, then own V pages
    const int newest = npages - 1 - pbeg;              // own index of the newest token's page (if in [0, nloc))
    const T *K = reinterpret_cast<const T *>(kv.k);
    const T *V = reinterpret_cast<const T *>(kv.v);
    const int *bt = kv.block_table + (long)seq * kv.max_pages + pbeg;
    auto page_src = [&](int u) -> const T * {
        const int p = u < nloc ? u : u - nloc;
        return (u < nloc ? K : V) + ((long)pgs[p] * kv.kv_heads + kvh) * (long)kAttnPage * D;
    };
    auto issue = [&](int u) {
        const int sl = u % S;
        mbar_expect_tx(bars + sl, kPageBytes);
        bulk_g2s(ring + sl * kPageBytes, page_src(u), kPageBytes, bars + sl);
    };
    auto is_newest = [&](int u) { return (u < nloc ? u : u - nloc) == newest; };
    if (tid < S) mbar_init(bars + tid, 1);
    if (early)
        for (int i = tid; i < nloc; i += 128) pgs[i] = bt[i];
    mbar_fence_init();
    __syncthreads();
    const int first = min(S, total);
    if (tid == 0 && early) {
        // decode: pages other than the newest token's were written by earlier launches
        for (int u = 0; u < first; ++u)
            if (!is_newest(u)) issue(u);
        for (int u = first; u < total; ++u)
            if (!is_newest(u))
                asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(page_src(u)),
                             "r"((uint32_t)kPageBytes)
                             : "memory");
    }
    pdl_wait();
    pdl_trigger();
    tl.mark(104, npages, G);
    if (!early) {
        for (int i = tid; i < nloc; i += 128) pgs[i] = bt[i];
        __syncthreads();
    }
    if (tid == 0)
        for (int u = 0; u < first; ++u)
            if (!early || is_newest(u)) issue(u);
    stage_q<T, D>(qs, q + (long)row * q_rs + (long)kvh * G * D, G);
    __syncthreads();
    tl.phase(0);  // q staged
    uint32_t qb[D / 16][2];
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
        qb[kk][0] = *reinterpret_cast<const uint32_t *>(qs + g * D + kk * 16 + 2 * t);
        qb[kk][1] = *reinterpret_cast<const uint32_t *>(qs + g * D + kk * 16 + 2 * t + 8);
    }

    // ---- 1: own scores, rounded to T, and the own row max per head
    float mx0 = -INFINITY, mx1 = -INFINITY;  // heads 2t, 2t+1
    bool ok = true;
    for (int p = 0; p < nloc; ++p) {
        const int slot = p % S;
        if (!mbar_wait_bounded(bars + slot, (p / S) & 1, err, 3)) ok = false;
        const T *kt = reinterpret_cast<const T *>(ring + slot * kPageBytes) + warp * 16 * D;
        float c[4] = {0.f, 0.f, 0.f, 0.f};
        if (ok) {
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
                uint32_t a0, a1, a2, a3;
                ldsm_x4(smem_u32(kt + (lane & 15) * D + kk * 16 + (lane >> 4) * 8), a0, a1, a2, a3);
                mma16<T>(c, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
            }
        }
        const int j0 = p * kAttnPage + warp * 16 + g;  // own key index
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int j = j0 + (i >> 1) * 8, h = 2 * t + (i & 1);
            const bool valid = (pbeg * kAttnPage + j) < L;
            const float sv = valid ? round_to<T>(c[i]) : -INFINITY;
            sc[h * lpad + j] = from_float<T>(valid ? sv : 0.f);
            if (i & 1)
                mx1 = fmaxf(mx1, sv * scale);
            else
                mx0 = fmaxf(mx0, sv * scale);
        }
        __syncthreads();  // everyone is done with this slot
        if (tid == 0 && p + S < total) issue(p + S);
    }
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
    }
    if (g == 0) {
        red[(2 * t) * 4 + warp] = mx0;
        red[(2 * t + 1) * 4 + warp] = mx1;
    }
    __syncthreads();
    cluster_wait();  // every CTA of the cluster runs
    if (tid < CS * 8) {
        const int h = tid & 7;
        const float m = fmaxf(fmaxf(red[h * 4], red[h * 4 + 1]), fmaxf(red[h * 4 + 2], red[h * 4 + 3]));
        st_cluster_f32(xm + z * 8 + h, tid >> 3, m);
    }
    cluster_arrive();
    cluster_wait();
    tl.phase(1);  // maxima exchanged
    // ---- 2: numerators in place and the own exponent sums; thread -> (head h, keys i0, i0 + 16, ...)
    const int h = tid >> 4, i0 = tid & 15;
    float M = -INFINITY;
    for (int zz = 0; zz < CS; ++zz) M = fmaxf(M, xm[zz * 8 + h]);
    T *srow = sc + h * lpad;
    const int nkeys = min(nloc * kAttnPage, max(0, L - pbeg * kAttnPage));  // own keys at or before pos
    float lsum = 0.f;
    for (int j0 = i0; j0 < nloc * kAttnPage; j0 += 16 * 8) {
        float e[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int j = j0 + 16 * u;
            e[u] = j < nkeys && h < G ? to_float(srow[j]) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int j = j0 + 16 * u;
            if (j < nkeys && h < G) {
                e[u] = expf(e[u] * scale - M);
                lsum += e[u];
            }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (j0 + 16 * u < nloc * kAttnPage) srow[j0 + 16 * u] = from_float<T>(e[u]);
    }
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
    if (i0 < CS) st_cluster_f32(xl + z * 8 + h, i0, lsum);
    cluster_arrive();
    cluster_wait();
    tl.phase(2);  // sums exchanged
    float sum = 0.f;
    for (int zz = 0; zz < CS; ++zz) sum += xl[zz * 8 + h];
    const float inv = 1.0f / sum;
    if (h < G)
        for (int j0 = i0; j0 < nkeys; j0 += 16 * 8) {
            float e[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (j0 + 16 * u < nkeys) e[u] = to_float(srow[j0 + 16 * u]);
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (j0 + 16 * u < nkeys) srow[j0 + 16 * u] = from_float<T>(e[u] * inv);
        }
    __syncthreads();

    // ---- 3: own partial O^T = V^T . P^T; warp w owns d-tiles w, w + 4
    constexpr int kDT = D / 16;
    constexpr int kA = kDT > 4 ? 2 : 1;
    float o[kA][4];
#pragma unroll
    for (int a = 0; a < kA; ++a) o[a][0] = o[a][1] = o[a][2] = o[a][3] = 0.f;
    for (int p = 0; p < nloc; ++p) {
        const int u = nloc + p, slot = u % S;
        if (!mbar_wait_bounded(bars + slot, (u / S) & 1, err, 3)) ok = false;
        if (p == newest && L % kAttnPage) {
            // rows past the sequence end hold stale cache bytes; their P is 0, but 0 * NaN is NaN
            T *vw = reinterpret_cast<T *>(ring + slot * kPageBytes);
            const int r0 = L - (pbeg + p) * kAttnPage;
            for (int i = tid; i < (kAttnPage - r0) * D; i += 128) vw[r0 * D + i] = from_float<T>(0.f);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncthreads();
        }
        const T *vt = reinterpret_cast<const T *>(ring + slot * kPageBytes);
        if (ok) {
#pragma unroll
            for (int ks = 0; ks < kAttnPage / 16; ++ks) {
                const int key0 = p * kAttnPage + ks * 16;
                const uint32_t b0 = *reinterpret_cast<const uint32_t *>(sc + g * lpad + key0 + 2 * t);
                const uint32_t b1 = *reinterpret_cast<const uint32_t *>(sc + g * lpad + key0 + 2 * t + 8);
#pragma unroll
                for (int a = 0; a < kA; ++a) {
                    const int d0 = (warp + 4 * a) * 16;
                    if (d0 < D) {
                        const int mi = lane >> 3, r = lane & 7;
                        const T *addr = vt + (ks * 16 + r + (mi >> 1) * 8) * D + d0 + (mi & 1) * 8;
                        uint32_t a0, a1, a2, a3;
                        ldsm_x4_t(smem_u32(addr), a0, a1, a2, a3);
                        mma16<T>(o[a], a0, a1, a2, a3, b0, b1);
                    }
                }
            }
        }
        __syncthreads();
        if (tid == 0 && u + S < total) issue(u + S);
    }
    tl.phase(3);  // own P.V
    // o[a]: rows d0 + g, d0 + g + 8; columns (heads) 2t, 2t + 1 -> owners
#pragma unroll
    for (int a = 0; a < kA; ++a) {
        const int d0 = (warp + 4 * a) * 16;
        if (d0 >= D) continue;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int d = d0 + g + (i >> 1) * 8, hh = 2 * t + (i & 1);
            if (hh < G) {
                const int e = hh * D + d;
                st_cluster_f32(xo + z * per + e / CS, e % CS, o[a][i]);
            }
        }
    }
    cluster_arrive();
    cluster_wait();
    // owned elements e = z, z + CS, ...: partials added in z order
    T *orow = out + (long)row * out_rs + (long)kvh * G * D;
    for (int e = z + tid * CS; e < G * D; e += 128 * CS) {
        float acc = 0.f;
        for (int zz = 0; zz < CS; ++zz) acc += xo[zz * per + e / CS];
        orow[e] = from_float<T>(acc);
    }
}

// ---------------------------------------------------------------- split-K decode attention
// For few (row, kv head) pairs and long contexts the pages are split over
// gridDim.z CTAs in two launches with the reference's rounding points intact:
//   scores:  s_j = T(q . k_j) of this split's keys -> global score rows, the
//            split's max m_z of s_j * scale per head and l_z = sum of
//            exp(s_j * scale - m_z) over its keys; the last CTA of the (row,
//            head) forms M = max m_z and sum = sum_z l_z exp(m_z - M) in split
//            order (the same softmax sum, factored by split);
//   pv:      every split CTA takes P_j = T(T(exp(s_j * scale - M)) / sum) for
//            its keys, multiplies its own V pages, writes an fp32 partial, and
//            the last CTA of the (row, head) adds the partials in split order
//            and stores T(o).

template <typename T, int D>
__global__ void __launch_bounds__(128) attn_split_scores_kernel(const T *__restrict__ q, long q_rs,
                                                                const int *__restrict__ seq_of_row,
                                                                const int *__restrict__ pos_of_row, KVPaged kv, int G,
                                                                int pps, int lpad, float scale, T *__restrict__ S,
                                                                float *__restrict__ mpart, float *__restrict__ minv,
                                                                int *__restrict__ counter, int *err, int early) {
    Timeline tl;
    constexpr int kPageBytes = kAttnPage * D * 2;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *ring = smem;
    uint64_t *bars = reinterpret_cast<uint64_t *>(ring + kAttnSlots * kPageBytes);
    float *red = reinterpret_cast<float *>(bars + kAttnSlots);  // [8][4]
    T *qs = reinterpret_cast<T *>(red + 32);                     // [8][D]
    const int kvh = blockIdx.x, row = blockIdx.y, z = blockIdx.z, nz = gridDim.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int seq = seq_of_row[row], pos = pos_of_row[row];
    const int L = pos + 1;
    const int npages = (L + kAttnPage - 1) / kAttnPage;
    const int p0 = z * pps, p1 = min(p0 + pps, npages);
    const int n = p1 > p0 ? p1 - p0 : 0;
    const T *K = reinterpret_cast<const T *>(kv.k);
    // decode: the newest page's id is read before the wait too (the block
    // table is not written by the producing kernel)
    const int *bt = kv.block_table + (long)seq * kv.max_pages;
    const long pg_last = early && tid == 0 && n > 0 && p1 == npages ? bt[npages - 1] : -1;
    auto page_src = [&](int i) -> const T * {
        const long pg = pg_last >= 0 && p0 + i == npages - 1 ? pg_last : bt[p0 + i];
        return K + (pg * kv.kv_heads + kvh) * (long)kAttnPage * D;
    };
    if (tid < kAttnSlots) mbar_init(bars + tid, 1);
    mbar_fence_init();
    __syncthreads();
    int issued = 0;
    if (tid == 0 && early)  // decode: pages before the newest one were written by earlier launches
        for (; issued < kAttnSlots && issued < n && p0 + issued < npages - 1; ++issued) {
            mbar_expect_tx(bars + issued, kPageBytes);
            bulk_g2s(ring + issued * kPageBytes, page_src(issued), kPageBytes, bars + issued);
        }
    pdl_wait();
    pdl_trigger();
    tl.mark(101, npages, nz);
    if (tid == 0)
        for (; issued < kAttnSlots && issued < n; ++issued) {
            mbar_expect_tx(bars + issued, kPageBytes);
            bulk_g2s(ring + issued * kPageBytes, page_src(issued), kPageBytes, bars + issued);
        }
    const T *qrow = q + (long)row * q_rs + (long)kvh * G * D;
    stage_q<T, D>(qs, qrow, G);
    __syncthreads();
    uint32_t qb[D / 16][2];
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
        qb[kk][0] = *reinterpret_cast<const uint32_t *>(qs + g * D + kk * 16 + 2 * t);
        qb[kk][1] = *reinterpret_cast<const uint32_t *>(qs + g * D + kk * 16 + 2 * t + 8);
    }
    T *srow = S + ((long)row * kv.kv_heads + kvh) * 8 * lpad;
    T *own = qs + 8 * D;  // [8][pps * 64] this split's scores
    const int wl = pps * kAttnPage;
    float mx0 = -INFINITY, mx1 = -INFINITY;
    bool ok = true;
    for (int i = 0; i < n; ++i) {
        const int slot = i % kAttnSlots;
        if (!mbar_wait_bounded(bars + slot, (i / kAttnSlots) & 1, err, 4)) ok = false;
        const T *kt = reinterpret_cast<const T *>(ring + slot * kPageBytes) + warp * 16 * D;
        float c[4] = {0.f, 0.f, 0.f, 0.f};
        if (ok) {
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
                uint32_t a0, a1, a2, a3;
                ldsm_x4(smem_u32(kt + (lane & 15) * D + kk * 16 + (lane >> 4) * 8), a0, a1, a2, a3);
                mma16<T>(c, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
            }
        }
        const int k0 = (p0 + i) * kAttnPage + warp * 16 + g;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int key = k0 + (j >> 1) * 8, h = 2 * t + (j & 1);
            const float sv = key < L ? round_to<T>(c[j]) : -INFINITY;
            srow[(long)h * lpad + key] = from_float<T>(key < L ? sv : 0.f);
            own[h * wl + key - p0 * kAttnPage] = from_float<T>(key < L ? sv : 0.f);
            if (j & 1)
                mx1 = fmaxf(mx1, sv * scale);
            else
                mx0 = fmaxf(mx0, sv * scale);
        }
        __syncthreads();
        if (tid == 0 && issued < n) {
            const int sl = issued % kAttnSlots;
            mbar_expect_tx(bars + sl, kPageBytes);
            bulk_g2s(ring + sl * kPageBytes, page_src(issued), kPageBytes, bars + sl);
            ++issued;
        }
    }
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
    }
    if (g == 0) {
        red[(2 * t) * 4 + warp] = mx0;
        red[(2 * t + 1) * 4 + warp] = mx1;
    }
    __syncthreads();
    const long rh = (long)row * kv.kv_heads + kvh;
    // this split's max and sum of exp(s * scale - max) per head over its own keys
    __shared__ float s_m[8];
    if (tid < 8) s_m[tid] = fmaxf(fmaxf(red[tid * 4], red[tid * 4 + 1]), fmaxf(red[tid * 4 + 2], red[tid * 4 + 3]));
    __syncthreads();
    {
        const int h = tid >> 4, i0 = tid & 15;  // 16 threads per head, keys i0, i0 + 16, ...
        const float mz = s_m[h];
        float lsum = 0.f;
        for (int j0 = i0; j0 < n * kAttnPage; j0 += 16 * 8) {
            float e[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int jj = j0 + 16 * u;
                e[u] = jj < n * kAttnPage && p0 * kAttnPage + jj < L && h < G ? to_float(own[h * wl + jj]) : 0.f;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int jj = j0 + 16 * u;
                if (jj < n * kAttnPage && p0 * kAttnPage + jj < L && h < G) lsum += expf(e[u] * scale - mz);
            }
        }
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
        if (i0 == 0) {
            mpart[(rh * nz + z) * 16 + h] = mz;
            mpart[(rh * nz + z) * 16 + 8 + h] = lsum;
        }
    }
    // the last split of this (row, head) combines the splits' (max, sum) pairs
    // in split order: M = max_z m_z, sum = sum_z l_z exp(m_z - M)
    __shared__ int last;
    __threadfence();
    __syncthreads();
    tl.phase(0);  // scores of this split
    if (tid == 0) last = atomicAdd(counter + rh, 1) == nz - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    // all splits' (max, sum) pairs into the page ring (free now) in one round trip
    float *pairs = reinterpret_cast<float *>(ring);  // [nz][16]
    {
        const float4 *src = reinterpret_cast<const float4 *>(mpart + rh * nz * 16);
        for (int i0 = tid; i0 < nz * 4; i0 += 4 * 128) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (i0 + u * 128 < nz * 4) v[u] = __ldcg(src + i0 + u * 128);
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (i0 + u * 128 < nz * 4) reinterpret_cast<float4 *>(pairs)[i0 + u * 128] = v[u];
        }
    }
    __syncthreads();
    if (tid < 8) {
        float M = -INFINITY;
        for (int zz = 0; zz < nz; ++zz) M = fmaxf(M, pairs[zz * 16 + tid]);
        float sum = 0.f;
        for (int zz = 0; zz < nz; ++zz) {
            const float l = pairs[zz * 16 + 8 + tid];
            if (l > 0.f) sum += l * expf(pairs[zz * 16 + tid] - M);
        }
        minv[rh * 16 + 2 * tid] = M;
        minv[rh * 16 + 2 * tid + 1] = 1.0f / sum;
    }
    if (tid == 0) counter[rh] = 0;
    tl.phase(2);  // normaliser
}

template <typename T, int D>
__global__ void __launch_bounds__(128) attn_split_pv_kernel(T *__restrict__ out, long out_rs,
                                                            const int *__restrict__ seq_of_row,
                                                            const int *__restrict__ pos_of_row, KVPaged kv, int G,
                                                            int pps, int lpad, float scale, const T *__restrict__ S,
                                                            const float *__restrict__ minv, float *__restrict__ opart,
                                                            int *__restrict__ counter, int *err, int early) {
    Timeline tl;
    constexpr int kPageBytes = kAttnPage * D * 2;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *ring = smem;
    uint64_t *bars = reinterpret_cast<uint64_t *>(ring + kAttnSlots * kPageBytes);
    T *pl = reinterpret_cast<T *>(bars + kAttnSlots);  // [8][pps * 64] this split's P
    __shared__ int last;
    const int kvh = blockIdx.x, row = blockIdx.y, z = blockIdx.z, nz = gridDim.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int seq = seq_of_row[row], pos = pos_of_row[row];
    const int L = pos + 1;
    const int npages = (L + kAttnPage - 1) / kAttnPage;
    const int Lpad = npages * kAttnPage;
    const int p0 = z * pps, p1 = min(p0 + pps, npages);
    const int n = p1 > p0 ? p1 - p0 : 0;
    const int wl = pps * kAttnPage;  // row length of pl
    const T *V = reinterpret_cast<const T *>(kv.v);
    // decode: the newest page's id is read before the wait too (the block
    // table is not written by the producing kernel)
    const int *bt = kv.block_table + (long)seq * kv.max_pages;
    const long pg_last = early && tid == 0 && n > 0 && p1 == npages ? bt[npages - 1] : -1;
    auto page_src = [&](int i) -> const T * {
        const long pg = pg_last >= 0 && p0 + i == npages - 1 ? pg_last : bt[p0 + i];
        return V + (pg * kv.kv_heads + kvh) * (long)kAttnPage * D;
    };
    if (tid < kAttnSlots) mbar_init(bars + tid, 1);
    mbar_fence_init();
    __syncthreads();
    int issued = 0;
    if (tid == 0 && early)
        for (; issued < kAttnSlots && issued < n && p0 + issued < npages - 1; ++issued) {
            mbar_expect_tx(bars + issued, kPageBytes);
            bulk_g2s(ring + issued * kPageBytes, page_src(issued), kPageBytes, bars + issued);
        }
    pdl_wait();
    pdl_trigger();
    tl.mark(102, npages, nz);
    if (tid == 0)
        for (; issued < kAttnSlots && issued < n; ++issued) {
            mbar_expect_tx(bars + issued, kPageBytes);
            bulk_g2s(ring + issued * kPageBytes, page_src(issued), kPageBytes, bars + issued);
        }
    const long rh = (long)row * kv.kv_heads + kvh;
    // P of this split's keys: T(T(e_j) / sum) with the row's max and sum from the scores launch
    {
        const int h = tid >> 4, i0 = tid & 15;
        const T *sr = S + (rh * 8 + h) * lpad;
        const float M = minv[rh * 16 + 2 * h], inv = minv[rh * 16 + 2 * h + 1];
        for (int jj0 = i0; jj0 < n * kAttnPage; jj0 += 16 * 8) {  // eight loads in flight
            float sv[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int j = p0 * kAttnPage + jj0 + 16 * u;
                sv[u] = jj0 + 16 * u < n * kAttnPage && j < L && h < G ? to_float(sr[j]) : 0.f;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int jj = jj0 + 16 * u, j = p0 * kAttnPage + jj;
                if (jj >= n * kAttnPage) continue;
                float pv = 0.f;
                if (j < L && h < G)
                    pv = to_float(from_float<T>(to_float(from_float<T>(expf(sv[u] * scale - M))) * inv));
                pl[h * wl + jj] = from_float<T>(pv);
            }
        }
    }
    __syncthreads();
    tl.phase(0);  // P of this split
    constexpr int kDT = D / 16;
    constexpr int kNA = kDT > 4 ? 2 : 1;
    float o[kNA][4];
#pragma unroll
    for (int a = 0; a < kNA; ++a) o[a][0] = o[a][1] = o[a][2] = o[a][3] = 0.f;
    bool ok = true;
    for (int i = 0; i < n; ++i) {
        const int slot = i % kAttnSlots;
        if (!mbar_wait_bounded(bars + slot, (i / kAttnSlots) & 1, err, 5)) ok = false;
        if (p0 + i == npages - 1 && L % kAttnPage) {
            // rows past the sequence end hold stale cache bytes; their P is 0, but 0 * NaN is NaN
            T *vw = reinterpret_cast<T *>(ring + slot * kPageBytes);
            const int r0 = L - (p0 + i) * kAttnPage;
            for (int e = tid; e < (kAttnPage - r0) * D; e += 128) vw[r0 * D + e] = from_float<T>(0.f);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncthreads();
        }
        const T *vt = reinterpret_cast<const T *>(ring + slot * kPageBytes);
        if (ok) {
#pragma unroll
            for (int ks = 0; ks < kAttnPage / 16; ++ks) {
                const int key0 = i * kAttnPage + ks * 16;
                const uint32_t b0 = *reinterpret_cast<const uint32_t *>(pl + g * wl + key0 + 2 * t);
                const uint32_t b1 = *reinterpret_cast<const uint32_t *>(pl + g * wl + key0 + 2 * t + 8);
#pragma unroll
                for (int a = 0; a < kNA; ++a) {
                    const int d0 = (warp + 4 * a) * 16;
                    const int mi = lane >> 3, r = lane & 7;
                    const T *addr = vt + (ks * 16 + r + (mi >> 1) * 8) * D + d0 + (mi & 1) * 8;
                    uint32_t a0, a1, a2, a3;
                    ldsm_x4_t(smem_u32(addr), a0, a1, a2, a3);
                    mma16<T>(o[a], a0, a1, a2, a3, b0, b1);
                }
            }
        }
        __syncthreads();
        if (tid == 0 && issued < n) {
            const int sl = issued % kAttnSlots;
            mbar_expect_tx(bars + sl, kPageBytes);
            bulk_g2s(ring + sl * kPageBytes, page_src(issued), kPageBytes, bars + sl);
            ++issued;
        }
    }
    // partial O^T of this split: rows d, columns (heads) 2t, 2t + 1
    float *op = opart + (rh * nz + z) * 8 * D;
#pragma unroll
    for (int a = 0; a < kNA; ++a) {
        const int d0 = (warp + 4 * a) * 16;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int d = d0 + g + (i >> 1) * 8, hh = 2 * t + (i & 1);
            op[hh * D + d] = o[a][i];
        }
    }
    __threadfence();
    __syncthreads();
    tl.phase(1);  // partial of this split
    if (tid == 0) last = atomicAdd(counter + rh, 1) == nz - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    T *orow = out + (long)row * out_rs + (long)kvh * G * D;
    for (int i4 = tid; i4 < G * D / 4; i4 += 128) {
        // four outputs per thread, partials added in split order, sixteen loads in flight
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int z0 = 0; z0 < nz; z0 += 16) {
            float4 v[16];
#pragma unroll
            for (int u = 0; u < 16; ++u)
                v[u] = z0 + u < nz ? __ldcg(reinterpret_cast<const float4 *>(opart + (rh * nz + z0 + u) * 8 * D) + i4)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int u = 0; u < 16; ++u)
                if (z0 + u < nz) {
                    acc.x += v[u].x;
                    acc.y += v[u].y;
                    acc.z += v[u].z;
                    acc.w += v[u].w;
                }
        }
        orow[4 * i4] = from_float<T>(acc.x);
        orow[4 * i4 + 1] = from_float<T>(acc.y);
        orow[4 * i4 + 2] = from_float<T>(acc.z);
        orow[4 * i4 + 3] = from_float<T>(acc.w);
    }
    if (tid == 0) counter[rh] = 0;
    tl.phase(2);  // combined
}

// Both split-K passes in one launch: every split CTA computes its scores and
// its (max, sum) pair, publishes the pair and waits (bounded) until all splits
// of its (row, head) have published -- the grid is launched only when it fits
// on the GPU at once, so every split is resident -- then forms M and the sum
// itself from the pairs in split order (the same values the two-launch path's
// last CTA computes), turns its own scores (kept in shared memory) into P and
// multiplies its V pages, which it requested while waiting.  The last CTA of
// the (row, head) adds the partials in split order.  Same arithmetic, one
// dependent hand-over fewer, and no round trip of the scores through memory.
template <typename T, int D>
__global__ void __launch_bounds__(128) attn_split_fused_kernel(T *__restrict__ out, long out_rs, const T *__restrict__ q,
                                                               long q_rs, const int *__restrict__ seq_of_row,
                                                               const int *__restrict__ pos_of_row, KVPaged kv, int G,
                                                               int pps, float scale, float *__restrict__ mpart,
                                                               float *__restrict__ opart, int *__restrict__ counter,
                                                               int *__restrict__ counter_a, int *err, int early,
                                                               unsigned long long limit_ns) {
    Timeline tl;
    constexpr int kPageBytes = kAttnPage * D * 2;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *ring = smem;
    uint64_t *bars = reinterpret_cast<uint64_t *>(ring + kAttnSlots * kPageBytes);
    float *red = reinterpret_cast<float *>(bars + kAttnSlots);  // [8][4]
    float *minv = red + 32;                                     // [8][2]: M, 1 / sum
    T *qs = reinterpret_cast<T *>(minv + 16);                   // [8][D]
    T *own = qs + 8 * D;                                        // [8][pps * 64] this split's scores, then P
    __shared__ int last, ok_s;
    const int kvh = blockIdx.x, row = blockIdx.y, z = blockIdx.z, nz = gridDim.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int seq = seq_of_row[row], pos = pos_of_row[row];
    const int L = pos + 1;
    const int npages = (L + kAttnPage - 1) / kAttnPage;
    const int p0 = z * pps, p1 = min(p0 + pps, npages);
    const int n = p1 > p0 ? p1 - p0 : 0;
    const int wl = pps * kAttnPage;
    const T *K = reinterpret_cast<const T *>(kv.k);
    const T *V = reinterpret_cast<const T *>(kv.v);
    const int *bt = kv.block_table + (long)seq * kv.max_pages;
    const long pg_last = early && tid == 0 && n > 0 && p1 == npages ? bt[npages - 1] : -1;
    // units 0..n-1: this split's K pages, n..2n-1: its V pages
    auto page_src = [&](int i) -> const T * {
        const int pi = i < n ? i : i - n;
        const long pg = pg_last >= 0 && p0 + pi == npages - 1 ? pg_last : bt[p0 + pi];
        return (i < n ? K : V) + (pg * kv.kv_heads + kvh) * (long)kAttnPage * D;
    };
    if (tid < kAttnSlots) mbar_init(bars + tid, 1);
    mbar_fence_init();
    __syncthreads();
    int issued = 0;
    if (tid == 0 && early)  // decode: pages before the newest one were written by earlier launches
        for (; issued < kAttnSlots && issued < n && p0 + issued < npages - 1; ++issued) {
            mbar_expect_tx(bars + issued, kPageBytes);
            bulk_g2s(ring + issued * kPageBytes, page_src(issued), kPageBytes, bars + issued);
        }
    pdl_wait();
    pdl_trigger();
    tl.mark(103, npages, nz);
    if (tid == 0)
        for (; issued < kAttnSlots && issued < 2 * n; ++issued) {
            mbar_expect_tx(bars + issued, kPageBytes);
            bulk_g2s(ring + issued * kPageBytes, page_src(issued), kPageBytes, bars + issued);
        }
    const T *qrow = q + (long)row * q_rs + (long)kvh * G * D;
    stage_q<T, D>(qs, qrow, G);
    __syncthreads();
    uint32_t qb[D / 16][2];
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
        qb[kk][0] = *reinterpret_cast<const uint32_t *>(qs + g * D + kk * 16 + 2 * t);
        qb[kk][1] = *reinterpret_cast<const uint32_t *>(qs + g * D + kk * 16 + 2 * t + 8);
    }
    // ---- scores of this split's keys, rounded to T, and the split's max per head
    float mx0 = -INFINITY, mx1 = -INFINITY;
    bool ok = true;
    int consumed = 0;
    for (int i = 0; i < n; ++i, ++consumed) {
        const int slot = consumed % kAttnSlots;
        if (!mbar_wait_bounded(bars + slot, (consumed / kAttnSlots) & 1, err, 4)) ok = false;
        const T *kt = reinterpret_cast<const T *>(ring + slot * kPageBytes) + warp * 16 * D;
        float c[4] = {0.f, 0.f, 0.f, 0.f};
        if (ok) {
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
                uint32_t a0, a1, a2, a3;
                ldsm_x4(smem_u32(kt + (lane & 15) * D + kk * 16 + (lane >> 4) * 8), a0, a1, a2, a3);
                mma16<T>(c, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
            }
        }
        const int k0 = (p0 + i) * kAttnPage + warp * 16 + g;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int key = k0 + (j >> 1) * 8, h = 2 * t + (j & 1);
            const float sv = key < L ? round_to<T>(c[j]) : -INFINITY;
            own[h * wl + key - p0 * kAttnPage] = from_float<T>(key < L ? sv : 0.f);
            if (j & 1)
                mx1 = fmaxf(mx1, sv * scale);
            else
                mx0 = fmaxf(mx0, sv * scale);
        }
        __syncthreads();  // the slot is free: request the next page (K, then this split's V pages)
        if (tid == 0 && issued < 2 * n) {
            const int sl = issued % kAttnSlots;
            mbar_expect_tx(bars + sl, kPageBytes);
            bulk_g2s(ring + sl * kPageBytes, page_src(issued), kPageBytes, bars + sl);
            ++issued;
        }
    }
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
    }
    if (g == 0) {
        red[(2 * t) * 4 + warp] = mx0;
        red[(2 * t + 1) * 4 + warp] = mx1;
    }
    __syncthreads();
    const long rh = (long)row * kv.kv_heads + kvh;
    __shared__ float s_m[8];
    if (tid < 8) s_m[tid] = fmaxf(fmaxf(red[tid * 4], red[tid * 4 + 1]), fmaxf(red[tid * 4 + 2], red[tid * 4 + 3]));
    __syncthreads();
    {
        const int h = tid >> 4, i0 = tid & 15;  // 16 threads per head, keys i0, i0 + 16, ...
        const float mz = s_m[h];
        float lsum = 0.f;
        for (int j0 = i0; j0 < n * kAttnPage; j0 += 16 * 8) {
            float e[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int jj = j0 + 16 * u;
                e[u] = jj < n * kAttnPage && p0 * kAttnPage + jj < L && h < G ? to_float(own[h * wl + jj]) : 0.f;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int jj = j0 + 16 * u;
                if (jj < n * kAttnPage && p0 * kAttnPage + jj < L && h < G) lsum += expf(e[u] * scale - mz);
            }
        }
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
        if (i0 == 0) {
            mpart[(rh * nz + z) * 16 + h] = mz;
            mpart[(rh * nz + z) * 16 + 8 + h] = lsum;
        }
    }
    __threadfence();
    __syncthreads();
    tl.phase(0);  // scores and pair of this split
    // ---- every split's pair: wait until all have published, then M and 1 / sum in split order
    if (tid == 0) {
        atomicAdd(counter_a + rh, 1);
        ok_s = 1;
        const uint64_t t0 = globaltimer_ns();
        while (*(volatile int *)(counter_a + rh) < nz) {
            if (globaltimer_ns() - t0 > limit_ns) {
                atomicCAS(err, 0, 6);
                ok_s = 0;
                break;
            }
            __nanosleep(64);
        }
        __threadfence();
    }
    __syncthreads();
    if (tid < 8) {
        float M = -INFINITY;
        for (int zz = 0; zz < nz; ++zz) M = fmaxf(M, __ldcg(mpart + (rh * nz + zz) * 16 + tid));
        float sum = 0.f;
        for (int zz = 0; zz < nz; ++zz) {
            const float l = __ldcg(mpart + (rh * nz + zz) * 16 + 8 + tid);
            if (l > 0.f) sum += l * expf(__ldcg(mpart + (rh * nz + zz) * 16 + tid) - M);
        }
        minv[2 * tid] = M;
        minv[2 * tid + 1] = 1.0f / sum;
    }
    __syncthreads();
    tl.phase(1);  // normaliser
    // ---- P of this split's keys: T(T(exp(s * scale - M)) * (1 / sum)), in place
    {
        const int h = tid >> 4, i0 = tid & 15;
        const float M = minv[2 * h], inv = minv[2 * h + 1];
        for (int jj = i0; jj < n * kAttnPage; jj += 16) {
            const int j = p0 * kAttnPage + jj;
            float pv = 0.f;
            if (j < L && h < G)
                pv = to_float(from_float<T>(to_float(from_float<T>(expf(to_float(own[h * wl + jj]) * scale - M))) * inv));
            own[h * wl + jj] = from_float<T>(pv);
        }
    }
    __syncthreads();
    // ---- P . V over this split's V pages
    constexpr int kDT = D / 16;
    constexpr int kNA = kDT > 4 ? 2 : 1;
    float o[kNA][4];
#pragma unroll
    for (int a = 0; a < kNA; ++a) o[a][0] = o[a][1] = o[a][2] = o[a][3] = 0.f;
    ok = ok && ok_s;
    for (int i = 0; i < n; ++i, ++consumed) {
        const int slot = consumed % kAttnSlots;
        if (!mbar_wait_bounded(bars + slot, (consumed / kAttnSlots) & 1, err, 5)) ok = false;
        if (p0 + i == npages - 1 && L % kAttnPage) {
            // rows past the sequence end hold stale cache bytes; their P is 0, but 0 * NaN is NaN
            T *vw = reinterpret_cast<T *>(ring + slot * kPageBytes);
            const int r0 = L - (p0 + i) * kAttnPage;
            for (int e = tid; e < (kAttnPage - r0) * D; e += 128) vw[r0 * D + e] = from_float<T>(0.f);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncthreads();
        }
        const T *vt = reinterpret_cast<const T *>(ring + slot * kPageBytes);
        if (ok) {
#pragma unroll
            for (int ks = 0; ks < kAttnPage / 16; ++ks) {
                const int key0 = i * kAttnPage + ks * 16;
                const uint32_t b0 = *reinterpret_cast<const uint32_t *>(own + g * wl + key0 + 2 * t);
                const uint32_t b1 = *reinterpret_cast<const uint32_t *>(own + g * wl + key0 + 2 * t + 8);
#pragma unroll
                for (int a = 0; a < kNA; ++a) {
                    const int d0 = (warp + 4 * a) * 16;
                    const int mi = lane >> 3, r = lane & 7;
                    const T *addr = vt + (ks * 16 + r + (mi >> 1) * 8) * D + d0 + (mi & 1) * 8;
                    uint32_t a0, a1, a2, a3;
                    ldsm_x4_t(smem_u32(addr), a0, a1, a2, a3);
                    mma16<T>(o[a], a0, a1, a2, a3, b0, b1);
                }
            }
        }
        __syncthreads();
        if (tid == 0 && issued < 2 * n) {
            const int sl = issued % kAttnSlots;
            mbar_expect_tx(bars + sl, kPageBytes);
            bulk_g2s(ring + sl * kPageBytes, page_src(issued), kPageBytes, bars + sl);
            ++issued;
        }
    }
    float *op = opart + (rh * nz + z) * 8 * D;
#pragma unroll
    for (int a = 0; a < kNA; ++a) {
        const int d0 = (warp + 4 * a) * 16;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int d = d0 + g + (i >> 1) * 8, hh = 2 * t + (i & 1);
            op[hh * D + d] = o[a][i];
        }
    }
    __threadfence();
    __syncthreads();
    tl.phase(2);  // partial of this split
    if (tid == 0) last = atomicAdd(counter + rh, 1) == nz - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    T *orow = out + (long)row * out_rs + (long)kvh * G * D;
    for (int i4 = tid; i4 < G * D / 4; i4 += 128) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int z0 = 0; z0 < nz; z0 += 16) {
            float4 v[16];
#pragma unroll
            for (int u = 0; u < 16; ++u)
                v[u] = z0 + u < nz ? __ldcg(reinterpret_cast<const float4 *>(opart + (rh * nz + z0 + u) * 8 * D) + i4)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int u = 0; u < 16; ++u)
                if (z0 + u < nz) {
                    acc.x += v[u].x;
                    acc.y += v[u].y;
                    acc.z += v[u].z;
                    acc.w += v[u].w;
                }
        }
        orow[4 * i4] = from_float<T>(acc.x);
        orow[4 * i4 + 1] = from_float<T>(acc.y);
        orow[4 * i4 + 2] = from_float<T>(acc.z);
        orow[4 * i4 + 3] = from_float<T>(acc.w);
    }
    // every split has passed both waits: the counters start from zero next launch
    if (tid == 0) {
        counter[rh] = 0;
        counter_a[rh] = 0;
    }
    tl.phase(3);  // combined
}

// Returns the launches made (0: not split; the caller launches one CTA per (row, kv head)).
template <typename T, int D>
int launch_split(T *out, long out_rs, const T *q, long q_rs, const int *seq_of_row, const int *pos_of_row,
                  int nrows, int max_len, const KVPaged &kv, int G, cudaStream_t s, bool pdl, bool early,
                  const AttnSplitWs &ws) {
    const char *env = getenv("WUKONG_SPLIT_ATTN");  // 0: one CTA per (row, kv head) always
    if (env && env[0] == '0') return 0;
    const int pages = (max_len + kAttnPage - 1) / kAttnPage;
    const int units = nrows * kv.kv_heads;
    int nz = (2 * g_rt.num_sms + units - 1) / units;
    if (nz > pages) nz = pages;
    if (nz > ws.max_splits) nz = ws.max_splits;
    // below 8 pages the second launch costs more than the split saves
    if (pages < 8 || nz < 2 || nrows > ws.max_rows || pages * kAttnPage > ws.lpad || kv.kv_heads > ws.max_kv_heads)
        return 0;
    const int pps = (pages + nz - 1) / nz;
    nz = (pages + pps - 1) / pps;
    if (nz < 2) return 0;
    const float scale = 1.0f / sqrtf((float)D);
    {
        // one launch when every split CTA fits on the GPU at once (they wait for each other)
        const char *one = getenv("WUKONG_SPLIT_ATTN_FUSED");
        const size_t smem_f = (size_t)kAttnSlots * kAttnPage * D * 2 + kAttnSlots * 8 + 48 * 4 + 8 * D * 2 +
                              (size_t)8 * pps * kAttnPage * 2;
        auto kf = attn_split_fused_kernel<T, D>;
        static int conf_f = 0;
        if (!(one && one[0] == '0') && (int)smem_f <= g_rt.max_smem_optin) {
            if ((int)smem_f > conf_f) {
                WK_CHECK(cudaFuncSetAttribute(kf, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_f));
                conf_f = (int)smem_f;
            }
            int per_sm = 0;
            WK_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kf, 128, smem_f));
            if ((long)kv.kv_heads * nrows * nz <= (long)per_sm * g_rt.num_sms) {
                cudaLaunchConfig_t cfg = {};
                cfg.gridDim = dim3(kv.kv_heads, nrows, nz);
                cfg.blockDim = dim3(128);
                cfg.stream = s;
                cfg.dynamicSmemBytes = smem_f;
                cudaLaunchAttribute attr[1];
                attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
                attr[0].val.programmaticStreamSerializationAllowed = 1;
                cfg.attrs = attr;
                cfg.numAttrs = (pdl && g_rt.pdl) ? 1 : 0;
                WK_CHECK(cudaLaunchKernelEx(&cfg, kf, out, out_rs, q, q_rs, seq_of_row, pos_of_row, kv, G, pps, scale,
                                            ws.mpart, ws.opart, ws.counter, ws.counter_a, g_rt.d_error,
                                            early ? 1 : 0, g_rt.wait_limit_ns));
                return 1;
            }
        }
    }
    const size_t smem_a = (size_t)kAttnSlots * kAttnPage * D * 2 + kAttnSlots * 8 + 32 * 4 + 8 * D * 2 +
                          (size_t)8 * pps * kAttnPage * 2;
    const size_t smem_b = (size_t)kAttnSlots * kAttnPage * D * 2 + kAttnSlots * 8 + (size_t)8 * pps * kAttnPage * 2;
    if ((int)smem_a > g_rt.max_smem_optin || (int)smem_b > g_rt.max_smem_optin) return 0;
    auto ka = attn_split_scores_kernel<T, D>;
    auto kb = attn_split_pv_kernel<T, D>;
    static int conf_a = 0, conf_b = 0;
    if ((int)smem_a > conf_a) {
        WK_CHECK(cudaFuncSetAttribute(ka, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_a));
        conf_a = (int)smem_a;
    }
    if ((int)smem_b > conf_b) {
        WK_CHECK(cudaFuncSetAttribute(kb, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_b));
        conf_b = (int)smem_b;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kv.kv_heads, nrows, nz);
    cfg.blockDim = dim3(128);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = (pdl && g_rt.pdl) ? 1 : 0;
    cfg.dynamicSmemBytes = smem_a;
    WK_CHECK(cudaLaunchKernelEx(&cfg, ka, q, q_rs, seq_of_row, pos_of_row, kv, G, pps, ws.lpad, scale,
                                (T *)ws.scores, ws.mpart, ws.minv, ws.counter_a, g_rt.d_error, early ? 1 : 0));
    cfg.dynamicSmemBytes = smem_b;
    cfg.numAttrs = g_rt.pdl ? 1 : 0;
    WK_CHECK(cudaLaunchKernelEx(&cfg, kb, out, out_rs, seq_of_row, pos_of_row, kv, G, pps, ws.lpad, scale,
                                (const T *)ws.scores, (const float *)ws.minv, ws.opart, ws.counter, g_rt.d_error,
                                early ? 1 : 0));
    return 2;
}

// Cluster decode attention (attn_cluster_kernel): CS CTAs per (row, KV head)
// with CS about 2 x SMs / pairs (at most 16 and at most the context's pages),
// pps pages per CTA, and a ring of S page slots (every own K and V page when
// they fit).  Returns 0 when the shape or the device does not take it.
template <typename T, int D>
int launch_cluster(T *out, long out_rs, const T *q, long q_rs, const int *seq_of_row, const int *pos_of_row,
                   int nrows, int max_len, const KVPaged &kv, int G, cudaStream_t s, bool pdl, bool early) {
    const char *env = getenv("WUKONG_CLUSTER_ATTN");  // 0: the split / one-CTA kernels
    if (env && env[0] == '0') return 0;
    const int pages = (max_len + kAttnPage - 1) / kAttnPage;
    const int pairs = nrows * kv.kv_heads;
    if (pages < 1 || pairs < 1) return 0;
    // The largest cluster: 16 CTAs for at most 4 pairs (tensor-parallel ranks hold 1-4 KV heads at batch
    // 1; one cluster then spreads a long context over many SMs), 8 otherwise -- a 16-CTA cluster of
    // large CTAs needs 16 free SMs of one processing cluster at once, and 8 such clusters started in
    // staggered waves (Llama-3.1-70B, batch 8, one KV head per rank: attention 34.5 -> 24.5 us per
    // layer with 8).  WUKONG_CLUSTER_MAX and WUKONG_CLUSTER_SLOTS (the deepest page ring) override.
    // (constant-initialised statics, read on first use: no guarded initialisation, so the static
    // archive needs no C++ runtime)
    static int cs_env = -1, s_max = -1;
    if (cs_env < 0) {
        const char *e = getenv("WUKONG_CLUSTER_MAX");
        const int v = e ? atoi(e) : 0;
        cs_env = v >= 1 && v <= kClusterMax ? v : 0;
        const char *f = getenv("WUKONG_CLUSTER_SLOTS");
        const int w = f ? atoi(f) : 0;
        s_max = w >= 2 && w <= 16 ? w : 16;
    }
    const int cs_max = cs_env ? cs_env : (pairs <= 4 ? kClusterMax : 8);
    int CS = (2 * g_rt.num_sms + pairs - 1) / pairs;
    if (CS < (pages + 47) / 48) CS = (pages + 47) / 48;  // at most 48 pages (their score rows) per CTA
    if (CS > cs_max) CS = cs_max;
    if (CS > pages) CS = pages;
    int pps = (pages + CS - 1) / CS;
    CS = (pages + pps - 1) / pps;
    int S = 2 * pps < s_max ? 2 * pps : s_max;
    while (S > 2 && cluster_smem(D, S, pps, CS).total > (size_t)g_rt.max_smem_optin) --S;
    const size_t smem = cluster_smem(D, S, pps, CS).total;
    if (smem > (size_t)g_rt.max_smem_optin) return 0;
    auto kern = attn_cluster_kernel<T, D>;
    static int configured = 0;
    if (!configured) {
        WK_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
        configured = 1;
    }
    static int smem_set = 0;
    if ((int)smem > smem_set) {
        WK_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        smem_set = (int)smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(CS * kv.kv_heads, nrows);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CS;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = (pdl && g_rt.pdl) ? 2 : 1;
    // a cluster of CS CTAs must fit on one GPU processing cluster
    int nclusters = 0;
    if (cudaOccupancyMaxActiveClusters(&nclusters, kern, &cfg) != cudaSuccess || nclusters < 1) {
        cudaGetLastError();
        return 0;
    }
    const float scale = 1.0f / sqrtf((float)D);
    WK_CHECK(cudaLaunchKernelEx(&cfg, kern, out, out_rs, q, q_rs, seq_of_row, pos_of_row, kv, G, CS, pps, S, scale,
                                g_rt.d_error, early ? 1 : 0));
    return 1;
}

template <typename T, int D>
void launch_decode_tc(T *out, long out_rs, const T *q, long q_rs, const int *seq_of_row, const int *pos_of_row,
                      int nrows, int max_len, const KVPaged &kv, int G, cudaStream_t s, bool pdl, const void *pf,
                      long pf_bytes, bool early) {
    const int Lpad = (max_len + kAttnPage - 1) / kAttnPage * kAttnPage;
    constexpr size_t kPageBytes = (size_t)kAttnPage * D * 2;
    const size_t fixed = kAttnMaxSlots * 8 + 64 * 4 + 8 * D * 2 + (size_t)8 * Lpad * 2 + (size_t)(Lpad / kAttnPage) * 4;
    int S = (int)(64 * 1024 / kPageBytes);
    if (S > kAttnMaxSlots) S = kAttnMaxSlots;
    if (S < kAttnMaxSlots || fixed + S * kPageBytes > (size_t)g_rt.max_smem_optin) S = kAttnSlots;
    const size_t smem = fixed + S * kPageBytes;
    if ((int)smem > g_rt.max_smem_optin) WK_PANIC("attention: context %d needs %zu B of shared memory", max_len, smem);
    auto kern = S == kAttnMaxSlots ? attn_decode_tc_kernel<T, D, kAttnMaxSlots> : attn_decode_tc_kernel<T, D, kAttnSlots>;
    static int configured[2] = {0, 0};
    if ((int)smem > configured[S == kAttnMaxSlots]) {
        WK_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        configured[S == kAttnMaxSlots] = (int)smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kv.kv_heads, nrows);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = (pdl && g_rt.pdl) ? 1 : 0;
    const float scale = 1.0f / sqrtf((float)D);
    WK_CHECK(cudaLaunchKernelEx(&cfg, kern, out, out_rs, q, q_rs, seq_of_row, pos_of_row, kv, G, Lpad, scale,
                                g_rt.d_error, pf, pf_bytes, early ? 1 : 0));
}

// ---------------------------------------------------------------- prefill (flash-style, tensor cores)
// Prefill rows: n consecutive query positions P..P+n-1 of each sequence over
// its paged K/V (64-token pages = 64-key blocks).  One CTA of 8 warps takes a
// tile of 128 "query rows" = 128 / G positions x the G query heads of one KV
// head (position-major), so every K/V block it loads serves all 128 rows; each
// warp owns 16 rows and keeps Q, the scores and O in mma.sync fragments.
// Two passes over the key blocks keep the reference's rounding points exactly
// (cuda.cu:767-852 with :673-765):
//   pass 1: s_j = T(q . k_j), the row max M of s_j * scale (exact) and the
//           softmax sum of exp(s_j * scale - M), accumulated per block with
//           the running-max rescaling (the same sum up to fp32 rounding order);
//   pass 2: s_j again (same products, same rounding), P_j =
//           T(T(exp(s_j * scale - M)) * (1 / sum)), O += P . V in fp32, and
//           finally T(O).
// K/V blocks stream through a 2-stage shared-memory ring by 16-byte cp.async
// copies into an XOR-swizzled layout (conflict-free ldmatrix); blocks wholly
// above a warp's positions are skipped (causal).
constexpr int kPfRows = 128;  // query rows per CTA (8 warps x 16)

__device__ __forceinline__ void cp_async16(void *dst, const void *src, int bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// byte offset of 16-byte chunk c of row r in a [rows][D] 16-bit tile (D >= 64)
template <int D> __device__ __forceinline__ uint32_t swz(int r, int c) {
    return (uint32_t)(r * (D * 2) + ((c ^ (r & 7)) << 4));
}
template <typename T> __device__ __forceinline__ uint32_t pack_t2(float a, float b) {
    T ha = from_float<T>(a), hb = from_float<T>(b);
    return (uint32_t)*reinterpret_cast<uint16_t *>(&ha) | ((uint32_t)*reinterpret_cast<uint16_t *>(&hb) << 16);
}

template <typename T, int D>
__global__ void __launch_bounds__(256, D == 64 ? 2 : 1)
    attn_prefill_kernel(T *__restrict__ out, long out_rs, const T *__restrict__ q, long q_rs, int n, int P, KVPaged kv,
                        int G, float scale) {
    constexpr int kCh = D / 8;                 // 16-byte chunks per row
    constexpr int kTile = kAttnPage * D * 2;   // bytes of one 64-key block
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *Qs = smem;                        // [128][D]
    uint8_t *Ks = Qs + kPfRows * D * 2;        // [2][64][D]
    uint8_t *Vs = Ks + 2 * kTile;              // [2][64][D]
    const int QP = kPfRows / G;
    const int tile = gridDim.x - 1 - blockIdx.x;  // the longest tiles first
    const int kvh = blockIdx.y, b = blockIdx.z;
    const int i0 = tile * QP;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int nkeys = P + min(n, i0 + QP);     // keys 0 .. the tile's last position
    const int nb = (nkeys + kAttnPage - 1) / kAttnPage;
    const T *K = reinterpret_cast<const T *>(kv.k);
    const T *V = reinterpret_cast<const T *>(kv.v);
    const int *bt = kv.block_table + (long)b * kv.max_pages;
    // q, K and V of these positions are written by the previous kernel
    pdl_wait();
    pdl_trigger();

    // positions of this thread's two rows (g, g + 8 of the warp's 16)
    const int r0 = warp * 16 + g, r1 = r0 + 8;
    const int pos0 = P + i0 + r0 / G, pos1 = P + i0 + r1 / G;
    const int wpos_max = P + i0 + (warp * 16 + 15) / G;  // the warp's last position

    // Q tile (rows past the sequence are zero)
    for (int idx = tid; idx < kPfRows * kCh; idx += 256) {
        const int r = idx / kCh, c = idx % kCh;
        const int i = i0 + r / G;
        const T *src = q + ((long)b * n + (i < n ? i : 0)) * q_rs + (long)(kvh * G + r % G) * D + c * 8;
        cp_async16(Qs + swz<D>(r, c), src, i < n ? 16 : 0);
    }
    auto load_block = [&](uint8_t *dst, const T *base, int kb) {
        const long pg = bt[kb];
        const T *blk = base + (pg * kv.kv_heads + kvh) * (long)kAttnPage * D;
        for (int idx = tid; idx < kAttnPage * kCh; idx += 256) {
            const int r = idx / kCh, c = idx % kCh;
            const bool ok = kb * kAttnPage + r < nkeys;  // unwritten keys arrive as zeros
            cp_async16(dst + swz<D>(r, c), blk + (long)r * D + c * 8, ok ? 16 : 0);
        }
    };
    load_block(Ks, K, 0);
    cp_async_commit();

    uint32_t qa[D / 16][4];
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    // scores of one block: c[nt][i]: n-tile nt (8 keys), i: (row g | g + 8) x (key 2t | 2t + 1)
    auto scores = [&](const uint8_t *kt, float (&c)[8][4]) {
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) c[nt][i] = 0.f;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
#pragma unroll
            for (int n2 = 0; n2 < 4; ++n2) {
                uint32_t b0, b1, b2, b3;
                const int key = n2 * 16 + (lane & 7) + ((lane >> 4) << 3);
                ldsm_x4(smem_u32(kt + swz<D>(key, 2 * kk + ((lane >> 3) & 1))), b0, b1, b2, b3);
                mma16<T>(c[2 * n2], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
                mma16<T>(c[2 * n2 + 1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
            }
    };

    // ---- pass 1: row max and softmax sum
    for (int kb = 0; kb < nb; ++kb) {
        if (kb + 1 < nb) {
            load_block(Ks + ((kb + 1) & 1) * kTile, K, kb + 1);
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        if (kb == 0) {
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk)
                ldsm_x4(smem_u32(Qs + swz<D>(warp * 16 + (lane & 15), 2 * kk + (lane >> 4))), qa[kk][0], qa[kk][1],
                        qa[kk][2], qa[kk][3]);
        }
        if (kb * kAttnPage <= wpos_max) {
            float c[8][4];
            scores(Ks + (kb & 1) * kTile, c);
            float bm0 = -INFINITY, bm1 = -INFINITY;
#pragma unroll
            for (int nt = 0; nt < 8; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int key = kb * kAttnPage + nt * 8 + 2 * t + (i & 1);
                    const bool hi = i >= 2;
                    const float sv = key <= (hi ? pos1 : pos0) ? round_to<T>(c[nt][i]) * scale : -INFINITY;
                    c[nt][i] = sv;
                    if (hi)
                        bm1 = fmaxf(bm1, sv);
                    else
                        bm0 = fmaxf(bm0, sv);
                }
#pragma unroll
            for (int o = 1; o < 4; o <<= 1) {
                bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, o));
                bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, o));
            }
            const float n0 = fmaxf(m0, bm0), n1 = fmaxf(m1, bm1);
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                s0 += expf(c[nt][0] - n0) + expf(c[nt][1] - n0);
                s1 += expf(c[nt][2] - n1) + expf(c[nt][3] - n1);
            }
            // rows with no key in this block keep their state (n = -inf only before any key)
            if (n0 != -INFINITY) {
                l0 = (m0 == -INFINITY ? 0.f : l0 * expf(m0 - n0)) + s0;
                m0 = n0;
            }
            if (n1 != -INFINITY) {
                l1 = (m1 == -INFINITY ? 0.f : l1 * expf(m1 - n1)) + s1;
                m1 = n1;
            }
        }
        __syncthreads();  // the stage is refilled next
    }
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, o);
        l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    }
    const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;

    // ---- pass 2: probabilities and O = P . V
    float o[D / 8][4];
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt)
#pragma unroll
        for (int i = 0; i < 4; ++i) o[dt][i] = 0.f;
    load_block(Ks, K, 0);
    load_block(Vs, V, 0);
    cp_async_commit();
    for (int kb = 0; kb < nb; ++kb) {
        if (kb + 1 < nb) {
            load_block(Ks + ((kb + 1) & 1) * kTile, K, kb + 1);
            load_block(Vs + ((kb + 1) & 1) * kTile, V, kb + 1);
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        if (kb * kAttnPage <= wpos_max) {
            float c[8][4];
            scores(Ks + (kb & 1) * kTile, c);
            uint32_t pa[4][4];  // P as the A operand of four 16-key slices
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                float pv[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int key = kb * kAttnPage + nt * 8 + 2 * t + (i & 1);
                    const bool hi = i >= 2;
                    pv[i] = 0.f;
                    if (key <= (hi ? pos1 : pos0)) {
                        const float e = expf(round_to<T>(c[nt][i]) * scale - (hi ? m1 : m0));
                        pv[i] = round_to<T>(e) * (hi ? inv1 : inv0);
                    }
                }
                pa[nt >> 1][(nt & 1) * 2 + 0] = pack_t2<T>(pv[0], pv[1]);
                pa[nt >> 1][(nt & 1) * 2 + 1] = pack_t2<T>(pv[2], pv[3]);
            }
            const uint8_t *vt = Vs + (kb & 1) * kTile;
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
#pragma unroll
                for (int d2 = 0; d2 < D / 16; ++d2) {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4_t(smem_u32(vt + swz<D>(ks * 16 + (lane & 15), 2 * d2 + (lane >> 4))), b0, b1, b2, b3);
                    // A: (row g, keys 2t..) (row g + 8, keys 2t..) (row g, keys 8 + 2t..) (row g + 8, keys 8 + 2t..)
                    mma16<T>(o[2 * d2], pa[ks][0], pa[ks][1], pa[ks][2], pa[ks][3], b0, b1);
                    mma16<T>(o[2 * d2 + 1], pa[ks][0], pa[ks][1], pa[ks][2], pa[ks][3], b2, b3);
                }
        }
        __syncthreads();
    }
    // O rows g, g + 8: T(o); position-major rows -> (position, head)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int r = h ? r1 : r0;
        const int i = i0 + r / G;
        if (i >= n) continue;
        T *orow = out + ((long)b * n + i) * out_rs + (long)(kvh * G + r % G) * D;
#pragma unroll
        for (int dt = 0; dt < D / 8; ++dt)
            *reinterpret_cast<uint32_t *>(orow + dt * 8 + 2 * t) = pack_t2<T>(o[dt][2 * h], o[dt][2 * h + 1]);
    }
}

template <typename T, int D>
void launch_prefill(T *out, long out_rs, const T *q, long q_rs, int batch, int n, int P, const KVPaged &kv, int G,
                    cudaStream_t s) {
    const size_t smem = (size_t)kPfRows * D * 2 + 4 * (size_t)kAttnPage * D * 2;
    auto kern = attn_prefill_kernel<T, D>;
    static bool configured = false;
    if (!configured) {
        WK_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        configured = true;
    }
    const int QP = kPfRows / G;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((n + QP - 1) / QP, kv.kv_heads, batch);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = g_rt.pdl ? 1 : 0;
    const float scale = 1.0f / sqrtf((float)D);
    WK_CHECK(cudaLaunchKernelEx(&cfg, kern, out, out_rs, q, q_rs, n, P, kv, G, scale));
}

}  // namespace

template <typename T>
int attention_paged(T *out, long out_rs, const T *q, long q_rs, const int *seq_of_row, const int *pos_of_row,
                     int nrows, int max_len, const PagedKV &c, int H, cudaStream_t s, bool pdl, const void *pf,
                     long pf_bytes, bool early, const AttnSplitWs *ws) {
    KVPaged kv{c.k, c.v, c.block_table, c.max_pages, c.page, c.kv_heads, c.hd};
    const int G = H / c.kv_heads;
    if constexpr (sizeof(T) == 2) {
        if (c.page == kAttnPage && G <= 8 && (c.hd == 64 || c.hd == 128) && ((uintptr_t)c.k % 16) == 0 &&
            ((uintptr_t)c.v % 16) == 0) {
            // decode rows: one cluster of CTAs per (row, KV head), unless one CTA each is asked for
            const char *one = getenv("WUKONG_SPLIT_ATTN");
            if (early && !(one && one[0] == '0')) {
                const int nc = c.hd == 64 ? launch_cluster<T, 64>(out, out_rs, q, q_rs, seq_of_row, pos_of_row, nrows,
                                                                   max_len, kv, G, s, pdl, early)
                                          : launch_cluster<T, 128>(out, out_rs, q, q_rs, seq_of_row, pos_of_row,
                                                                    nrows, max_len, kv, G, s, pdl, early);
                if (nc) return nc;
            }
            const int ns = !ws ? 0
                           : c.hd == 64 ? launch_split<T, 64>(out, out_rs, q, q_rs, seq_of_row, pos_of_row, nrows,
                                                              max_len, kv, G, s, pdl, early, *ws)
                                        : launch_split<T, 128>(out, out_rs, q, q_rs, seq_of_row, pos_of_row, nrows,
                                                               max_len, kv, G, s, pdl, early, *ws);
            if (ns) return ns;
            if (c.hd == 64)
                launch_decode_tc<T, 64>(out, out_rs, q, q_rs, seq_of_row, pos_of_row, nrows, max_len, kv, G, s, pdl,
                                        pf, pf_bytes, early);
            else
                launch_decode_tc<T, 128>(out, out_rs, q, q_rs, seq_of_row, pos_of_row, nrows, max_len, kv, G, s, pdl,
                                         pf, pf_bytes, early);
            return 1;
        }
    }
    launch_rows<T>(out, out_rs, q, q_rs, seq_of_row, pos_of_row, 1, nrows, max_len, kv, H, c.kv_heads, c.hd, s, pdl);
    return 1;
}
template int attention_paged<__half>(__half *, long, const __half *, long, const int *, const int *, int, int,
                                      const PagedKV &, int, cudaStream_t, bool, const void *, long, bool,
                                      const AttnSplitWs *);
template int attention_paged<__nv_bfloat16>(__nv_bfloat16 *, long, const __nv_bfloat16 *, long, const int *,
                                             const int *, int, int, const PagedKV &, int, cudaStream_t, bool,
                                             const void *, long, bool, const AttnSplitWs *);
template int attention_paged<float>(float *, long, const float *, long, const int *, const int *, int, int,
                                     const PagedKV &, int, cudaStream_t, bool, const void *, long, bool,
                                     const AttnSplitWs *);

template <typename T>
int attention_prefill_paged(T *out, long out_rs, const T *q, long q_rs, int batch, int n, int P, const PagedKV &c,
                            int H, cudaStream_t s) {
    if (batch <= 0 || n <= 0) return 0;
    KVPaged kv{c.k, c.v, c.block_table, c.max_pages, c.page, c.kv_heads, c.hd};
    const int G = H / c.kv_heads;
    if constexpr (sizeof(T) == 2) {
        if (c.page == kAttnPage && (G == 1 || G == 2 || G == 4 || G == 8) && (c.hd == 64 || c.hd == 128) &&
            ((uintptr_t)c.k % 16) == 0 && ((uintptr_t)c.v % 16) == 0 && ((uintptr_t)q % 16) == 0 && (q_rs % 8) == 0 &&
            ((uintptr_t)out % 4) == 0 && (out_rs % 2) == 0) {
            if (c.hd == 64)
                launch_prefill<T, 64>(out, out_rs, q, q_rs, batch, n, P, kv, G, s);
            else
                launch_prefill<T, 128>(out, out_rs, q, q_rs, batch, n, P, kv, G, s);
            return 1;
        }
    }
    return -1;  // the caller uses attention_paged
}
template int attention_prefill_paged<__half>(__half *, long, const __half *, long, int, int, int, const PagedKV &, int,
                                             cudaStream_t);
template int attention_prefill_paged<__nv_bfloat16>(__nv_bfloat16 *, long, const __nv_bfloat16 *, long, int, int, int,
                                                    const PagedKV &, int, cudaStream_t);

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

#ifdef WK_TIMELINE
void timeline_bind_attn(const TimelineBuf &b) { WK_CHECK(cudaMemcpyToSymbol(c_tl, &b, sizeof b)); }
#else
void timeline_bind_attn(const TimelineBuf &) {}
#endif

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
