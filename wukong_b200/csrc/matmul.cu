// cuda_matmul (cuda.h:7) and the shared matmul dispatcher.
//
// Reference semantics (cuda.cu:1095-1111, :270-341): out[M, N] = X[M, K] W[N, K]^T
// (+ bias) with T = float / bf16 / half chosen by the weight dtype; quantised
// weights are first dequantised to half.  Accumulation in fp32, one rounding to
// T at the store, bias added before that rounding (cuBLASLt BIAS epilogue).
//
// Dispatch: 16-bit and Q8_0 weights go to the dequant-fused GEMV (gemv.cu), up
// to 8 activation rows per pass.  F32 weights and shapes the GEMV does not take
// (K not a multiple of 16/32) use matmul_generic_kernel, a shared-memory tiled
// CUDA-core kernel with exact fp32 products.
#include "common.cuh"
#include "wukong_internal.cuh"

namespace wk {

namespace {

// weight element (n, k) with the reference's dequantise-to-half rounding
template <int WT> __device__ __forceinline__ float wload(const uint8_t *w, long rb, int n, int k);
template <> __device__ __forceinline__ float wload<kF32>(const uint8_t *w, long rb, int n, int k) {
    return reinterpret_cast<const float *>(w + n * rb)[k];
}
template <> __device__ __forceinline__ float wload<kF16>(const uint8_t *w, long rb, int n, int k) {
    return __half2float(reinterpret_cast<const __half *>(w + n * rb)[k]);
}
template <> __device__ __forceinline__ float wload<kBF16>(const uint8_t *w, long rb, int n, int k) {
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(w + n * rb)[k]);
}
template <> __device__ __forceinline__ float wload<kQ8_0>(const uint8_t *w, long rb, int n, int k) {
    const uint8_t *blk = w + n * rb + (k / 32) * 34;
    const __half s = __ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8)));
    return __half2float(__float2half_rn(__half2float(s) * (float)(int8_t)blk[2 + (k & 31)]));
}

constexpr int TM = 32, TN = 32, TK = 32;

template <typename T, int WT>
__global__ void __launch_bounds__(256) matmul_generic_kernel(T *__restrict__ out, const T *__restrict__ x,
                                                             const uint8_t *__restrict__ w, long rb,
                                                             const T *__restrict__ bias, int M, int K, int N) {
    __shared__ float xs[TM][TK + 1];
    __shared__ float ws[TN][TK + 1];
    const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;  // 16 x 16 threads, 2 x 2 outputs each
    float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
    for (int k0 = 0; k0 < K; k0 += TK) {
        for (int i = threadIdx.x; i < TM * TK; i += 256) {
            const int r = i / TK, c = i % TK;
            xs[r][c] = (m0 + r < M && k0 + c < K) ? to_float(x[(long)(m0 + r) * K + k0 + c]) : 0.f;
            ws[r][c] = (n0 + r < N && k0 + c < K) ? wload<WT>(w, rb, n0 + r, k0 + c) : 0.f;
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < TK; ++k) {
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int j = 0; j < 2; ++j) acc[i][j] += xs[ty + 16 * i][k] * ws[tx + 16 * j][k];
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int m = m0 + ty + 16 * i, n = n0 + tx + 16 * j;
            if (m < M && n < N) {
                float v = acc[i][j];
                if (bias) v += to_float(bias[n]);
                out[(long)m * N + n] = from_float<T>(v);
            }
        }
}

template <typename T, int WT>
void launch_generic(void *out, const void *x, const void *w, const void *bias, int M, int K, int N, cudaStream_t s) {
    long rb = WT == kQ8_0 ? (long)(K / 32) * 34 : (long)K * (WT == kF32 ? 4 : 2);
    dim3 grid((N + TN - 1) / TN, (M + TM - 1) / TM);
    matmul_generic_kernel<T, WT><<<grid, 256, 0, s>>>((T *)out, (const T *)x, (const uint8_t *)w, rb,
                                                      (const T *)bias, M, K, N);
    WK_CHECK_LAUNCH();
}

__global__ void fill_row_meta_kernel(int *seq, int *pos, int rows, int n, int pos0) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < rows) {
        seq[i] = i / n;
        pos[i] = pos0 + i % n;
    }
}

__global__ void fill_block_table_kernel(int *bt, int total, int pages) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < total) bt[i] = i;  // row b, page p -> b * pages + p
}

}  // namespace

void fill_row_meta(int *seq, int *pos, int rows, int n, int pos0, cudaStream_t s) {
    if (rows <= 0) return;
    fill_row_meta_kernel<<<(rows + 255) / 256, 256, 0, s>>>(seq, pos, rows, n, pos0);
    WK_CHECK_LAUNCH();
}

void fill_block_table(int *bt, int batch, int pages, cudaStream_t s) {
    int total = batch * pages;
    if (total <= 0) return;
    fill_block_table_kernel<<<(total + 255) / 256, 256, 0, s>>>(bt, total, pages);
    WK_CHECK_LAUNCH();
}

void matmul(void *out, const void *x, const void *w, const void *bias, int M, int K, int N, int wtype, int act,
            cudaStream_t s) {
    if (M <= 0 || N <= 0) return;
    const size_t es0 = act_size(act);
    if (M >= kTcMinRows && g_rt.tc_gemm && gemm_tc_supported(wtype, act, K, N, EPI_STORE, 0) &&
        ((uintptr_t)x % 16) == 0 && ((uintptr_t)w % 16) == 0 && ((size_t)K * es0) % 16 == 0 &&
        (wtype != kQ8_0 || ((size_t)(K / 32) * 34) % 16 == 0)) {
        GemmArgs a;
        a.w = (const uint8_t *)w;
        a.wtype = wtype;
        a.N = N;
        a.K = K;
        a.x = x;
        a.ldx = K;
        a.M = M;
        a.epi = EPI_STORE;
        a.out = out;
        a.ldo = N;
        a.bias = bias;
        gemm_tc(a, act, s);
        return;
    }
    if (gemv_supported(wtype, act, K)) {
        const size_t es = act_size(act);
        for (int m0 = 0; m0 < M; m0 += 8) {
            GemvArgs a;
            a.w = (const uint8_t *)w;
            a.wtype = wtype;
            a.N = N;
            a.K = K;
            a.x = (const char *)x + (size_t)m0 * K * es;
            a.ldx = K;
            a.M = M - m0 < 8 ? M - m0 : 8;
            a.epi = EPI_STORE;
            a.out = (char *)out + (size_t)m0 * N * es;
            a.ldo = N;
            a.bias = bias;
            gemv(a, act, s);
        }
        return;
    }
    switch (wtype) {
    case kF32:
        if (act != kF32) WK_PANIC("F32 weights need F32 activations");
        launch_generic<float, kF32>(out, x, w, bias, M, K, N, s);
        break;
    case kF16:
        launch_generic<__half, kF16>(out, x, w, bias, M, K, N, s);
        break;
    case kBF16:
        launch_generic<__nv_bfloat16, kBF16>(out, x, w, bias, M, K, N, s);
        break;
    case kQ8_0:
        if (K % 32) WK_PANIC("Q8_0 weights need K %% 32 == 0 (K=%d)", K);
        launch_generic<__half, kQ8_0>(out, x, w, bias, M, K, N, s);
        break;
    default:
        WK_PANIC("Unsupported quantization type: %s", (wtype >= 0 && wtype < kDTypeCount) ? kDTypes[wtype].name : "?");
    }
}

int linear(const GemvArgs &g, int rows, int act, cudaStream_t s, void *norm_scratch) {
    if (rows <= 0) return 0;
    const size_t es = act_size(act);
    const bool tc = rows >= kTcMinRows && g_rt.tc_gemm && g.epi != EPI_LOGITS &&
                    gemm_tc_supported(g.wtype, act, g.K, g.N, g.epi, g.F) && ((uintptr_t)g.w % 16) == 0 &&
                    (g.wtype != kQ8_0 || ((size_t)(g.K / 32) * 34) % 16 == 0) &&
                    (!g.norm_w || (norm_scratch && g.ldx == g.K && ((uintptr_t)norm_scratch % 16) == 0)) &&
                    (g.norm_w || (((uintptr_t)g.x % 16) == 0 && ((size_t)g.ldx * es) % 16 == 0));
    if (tc) {
        GemmArgs a;
        a.w = g.w;
        a.wtype = g.wtype;
        a.N = g.N;
        a.K = g.K;
        a.x = g.x;
        a.ldx = g.ldx;
        int n = 0;
        if (g.norm_w) {
            // the GEMM reads the normalised rows (same rounding as the GEMV prologue)
            if (act == kBF16)
                rmsnorm<__nv_bfloat16>((__nv_bfloat16 *)norm_scratch, (const __nv_bfloat16 *)g.x, g.norm_w, rows, g.K,
                                       g.eps, s);
            else
                rmsnorm<__half>((__half *)norm_scratch, (const __half *)g.x, g.norm_w, rows, g.K, g.eps, s);
            a.x = norm_scratch;
            a.ldx = g.K;
            ++n;
        }
        a.M = rows;
        a.epi = g.epi;
        a.out = g.out;
        a.ldo = g.ldo;
        a.bias = g.bias;
        a.res = g.res;
        a.ldr = g.ldr;
        a.nq = g.nq;
        a.nk = g.nk;
        a.hd = g.hd;
        a.freqs = g.freqs;
        a.pos = g.pos;
        a.seq = g.seq;
        a.kpool = g.kpool;
        a.vpool = g.vpool;
        a.block_table = g.block_table;
        a.max_pages = g.max_pages;
        a.page = g.page;
        a.kv_heads = g.kv_heads;
        a.F = g.F;
        a.err = g.err;
        a.pdl = g.pdl;
        gemm_tc(a, act, s);
        return n + 1;
    }
    int n = 0;
    for (int m0 = 0; m0 < rows; m0 += 8, ++n) {
        GemvArgs a = g;
        a.M = rows - m0 < 8 ? rows - m0 : 8;
        a.x = (const char *)g.x + (size_t)m0 * g.ldx * es;
        if (g.out && g.epi != EPI_LOGITS)
            a.out = (char *)g.out + (size_t)m0 * g.ldo * (g.epi == EPI_PARTIAL ? 4 : es);
        if (g.res) a.res = (const char *)g.res + (size_t)m0 * g.ldr * es;
        if (g.pos) a.pos = g.pos + m0;
        if (g.seq) a.seq = g.seq + m0;
        if (g.tokens) a.tokens = g.tokens + m0;
        if (g.best_val) {
            a.best_val = g.best_val + m0;
            a.best_key = g.best_key + m0;
        }
        if (m0) {
            a.pf = nullptr;
            a.pf_bytes = 0;
        }
        gemv(a, act, s);
    }
    return n;
}

}  // namespace wk

using namespace wk;

extern "C" {

// cuda.cu:1095-1111.  Activations are float for F32 weights, bf16 for BF16,
// half for F16 and Q8_0 (the reference reads them as half for every quantised
// dtype, cuda.cu:1105-1107).
void cuda_matmul(void *out, const void *inp, const void *weight, const void *bias, int row, int column, int oc,
                 int dtype) {
    ensure_init();
    if (dtype < 0 || dtype >= kDTypeCount) WK_PANIC("Unsupported quantization type: %d", dtype);
    if (dtype != kF32 && dtype != kF16 && dtype != kBF16 && dtype != kQ8_0 && dtype != kQ4_0)
        WK_PANIC("Unsupported quantization type: %s", kDTypes[dtype].name);
    if (dtype == kQ4_0 && column % 32) WK_PANIC("Q4_0 weights need K %% 32 == 0 (K=%d)", column);
    if (bias && ((uintptr_t)bias % 16)) WK_PANIC("bias must be aligned to 16 bytes");
    matmul(out, inp, weight, bias, row, column, oc, dtype, act_of(dtype), stream());
}

}  // extern "C"
