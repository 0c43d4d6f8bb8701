// Element-wise and row-wise ops of the C ABI: dequantise, embedding, rmsnorm,
// rope, swiglu, add, div, softmax, get_row, argmax, repeat_qkv.
//
// Each kernel keeps the reference's numerics (fp32 math, one rounding to the
// storage type T per stored value) but not its launch shapes: rows are handled
// by whole CTAs or warps with vectorised, coalesced accesses and no
// divisibility requirement on the row length.
#include "common.cuh"
#include "wukong_internal.cuh"

namespace wk {

// ------------------------------------------------------------ Q8_0 dequantise
// cuda.cu:389-421: out = (T)(float(scale) * q).  One warp per 32 blocks: the
// warp stages its 1088 contiguous bytes in shared memory with coalesced 4-byte
// loads (the 34-byte blocks are not 4-byte aligned), then each lane expands one
// block with 16-byte stores.
template <typename T>
__global__ void __launch_bounds__(256) dequant_q8_0_kernel(T *__restrict__ out, const uint8_t *__restrict__ in,
                                                           long nblocks) {
    __shared__ __align__(16) uint8_t stage[8][32 * kQ8Bytes + 4];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long b0 = ((long)blockIdx.x * 8 + warp) * 32;
    if (b0 >= nblocks) return;
    const int nb = (int)min((long)32, nblocks - b0);
    const uint8_t *src = in + b0 * kQ8Bytes;
    uint8_t *st = stage[warp];
    for (int i = lane; i < nb * kQ8Bytes; i += 32) st[i] = src[i];
    __syncwarp();
    if (lane < nb) {
        const uint8_t *blk = st + lane * kQ8Bytes;
        const float scale = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
        T *o = out + (b0 + lane) * kQ8Block;
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = from_float<T>(scale * (float)(int8_t)blk[2 + i]);
    }
}

template <typename T> void dequant_q8_0(T *out, const void *in, long nblocks, cudaStream_t s) {
    if (nblocks <= 0) return;
    long grid = (nblocks + 255) / 256;
    dequant_q8_0_kernel<T><<<(unsigned)grid, 256, 0, s>>>(out, (const uint8_t *)in, nblocks);
    WK_CHECK_LAUNCH();
}
template void dequant_q8_0<float>(float *, const void *, long, cudaStream_t);
template void dequant_q8_0<__half>(__half *, const void *, long, cudaStream_t);

// ------------------------------------------------------------ Q4_0 dequantise
// The reference dequantises only Q8_0 (cuda.cu:1006-1012) though its dtype table
// lists Q4_0 (cuda.cu:5-42); this applies its Q8_0 rule to GGUF Q4_0 blocks:
// out = (T)(float(d) * (n - 8)) for the stored nibble n (exact product).
template <typename T>
__global__ void __launch_bounds__(256) dequant_q4_0_kernel(T *__restrict__ out, const uint8_t *__restrict__ in,
                                                           long nblocks) {
    const long b = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    const uint8_t *blk = in + b * kQ4Bytes;
    const float d = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
    T *o = out + b * 32;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        o[i] = from_float<T>(d * (float)((int)(blk[2 + i] & 15) - 8));
        o[i + 16] = from_float<T>(d * (float)((int)(blk[2 + i] >> 4) - 8));
    }
}

template <typename T> void dequant_q4_0(T *out, const void *in, long nblocks, cudaStream_t s) {
    if (nblocks <= 0) return;
    dequant_q4_0_kernel<T><<<(unsigned)((nblocks + 255) / 256), 256, 0, s>>>(out, (const uint8_t *)in, nblocks);
    WK_CHECK_LAUNCH();
}
template void dequant_q4_0<float>(float *, const void *, long, cudaStream_t);
template void dequant_q4_0<__half>(__half *, const void *, long, cudaStream_t);

template <typename T>
__global__ void gather_q4_0_kernel(T *__restrict__ out, const int *__restrict__ ids, const uint8_t *__restrict__ table,
                                   int n, int col) {
    const int r = blockIdx.x;
    if (r >= n) return;
    const uint8_t *row = table + (size_t)ids[r] * (col / 32) * kQ4Bytes;
    for (int i = threadIdx.x; i < col; i += blockDim.x) {
        const uint8_t *blk = row + (i / 32) * kQ4Bytes;
        const float d = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
        const int j = i & 31;
        const int nib = j < 16 ? (blk[2 + j] & 15) : (blk[2 + j - 16] >> 4);
        out[(size_t)r * col + i] = from_float<T>(d * (float)(nib - 8));
    }
}

// ------------------------------------------------------------ embedding
// cuda.cu:238-252, :1232-1255: byte gather of whole rows for plain dtypes; for
// Q8_0 the gathered blocks are dequantised to half (fused here).
__global__ void gather_rows_kernel(uint8_t *__restrict__ out, const int *__restrict__ ids,
                                   const uint8_t *__restrict__ table, int n, size_t row_bytes) {
    const int r = blockIdx.x;
    if (r >= n) return;
    const uint8_t *src = table + (size_t)ids[r] * row_bytes;
    uint8_t *dst = out + (size_t)r * row_bytes;
    if ((row_bytes & 15) == 0 && (((uintptr_t)src | (uintptr_t)dst) & 15) == 0) {
        for (size_t i = threadIdx.x; i < row_bytes / 16; i += blockDim.x)
            reinterpret_cast<int4 *>(dst)[i] = reinterpret_cast<const int4 *>(src)[i];
    } else {
        for (size_t i = threadIdx.x; i < row_bytes; i += blockDim.x) dst[i] = src[i];
    }
}

template <typename T>
__global__ void gather_q8_0_kernel(T *__restrict__ out, const int *__restrict__ ids, const uint8_t *__restrict__ table,
                                   int n, int col) {
    const int r = blockIdx.x;
    if (r >= n) return;
    const int nb = col / kQ8Block;
    const uint8_t *row = table + (size_t)ids[r] * nb * kQ8Bytes;
    for (int i = threadIdx.x; i < col; i += blockDim.x) {
        const uint8_t *blk = row + (i / kQ8Block) * kQ8Bytes;
        const float scale = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
        out[(size_t)r * col + i] = from_float<T>(scale * (float)(int8_t)blk[2 + (i % kQ8Block)]);
    }
}

void embedding(void *out, const int *ids, const void *table, int n, int col, int dtype, int out_act, cudaStream_t s) {
    if (n <= 0) return;
    if (dtype == kQ8_0) {
        if (out_act == kF32)
            gather_q8_0_kernel<float><<<n, 256, 0, s>>>((float *)out, ids, (const uint8_t *)table, n, col);
        else
            gather_q8_0_kernel<__half><<<n, 256, 0, s>>>((__half *)out, ids, (const uint8_t *)table, n, col);
    } else if (dtype == kQ4_0) {
        if (out_act == kF32)
            gather_q4_0_kernel<float><<<n, 256, 0, s>>>((float *)out, ids, (const uint8_t *)table, n, col);
        else
            gather_q4_0_kernel<__half><<<n, 256, 0, s>>>((__half *)out, ids, (const uint8_t *)table, n, col);
    } else {
        const DTypeInfo &info = kDTypes[dtype];
        size_t row_bytes = (size_t)col / info.block_size * info.type_size;
        gather_rows_kernel<<<n, 128, 0, s>>>((uint8_t *)out, ids, (const uint8_t *)table, n, row_bytes);
    }
    WK_CHECK_LAUNCH();
}

// ------------------------------------------------------------ rmsnorm
// cuda.cu:533-601: y = (x * rsqrt(mean(x^2) + eps)) * w, w fp32.
template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_kernel(T *__restrict__ out, const T *__restrict__ in,
                                                      const float *__restrict__ w, int C, float eps) {
    __shared__ float red[32];
    const T *x = in + (size_t)blockIdx.x * C;
    float ss = 0.f;
    for (int i = threadIdx.x; i < C; i += blockDim.x) {
        float v = to_float(x[i]);
        ss += v * v;
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        v = warp_sum(v);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float s = rsqrtf(red[0] / (float)C + eps);
    T *o = out + (size_t)blockIdx.x * C;
    for (int i = threadIdx.x; i < C; i += blockDim.x) o[i] = from_float<T>((to_float(x[i]) * s) * w[i]);
}

template <typename T> void rmsnorm(T *out, const T *in, const float *w, int rows, int C, float eps, cudaStream_t s) {
    if (rows <= 0) return;
    rmsnorm_kernel<T><<<rows, 256, 0, s>>>(out, in, w, C, eps);
    WK_CHECK_LAUNCH();
}
template void rmsnorm<float>(float *, const float *, const float *, int, int, float, cudaStream_t);
template void rmsnorm<__half>(__half *, const __half *, const float *, int, int, float, cudaStream_t);
template void rmsnorm<__nv_bfloat16>(__nv_bfloat16 *, const __nv_bfloat16 *, const float *, int, int, float,
                                     cudaStream_t);

// ------------------------------------------------------------ rope
// cuda.cu:207-236: rotate interleaved pairs of the first `nrot` heads of each row
// (of `heads_per_row` heads); row r of batch b uses freqs[(pos0 + r) * HS].
template <typename T>
__global__ void rope_kernel(T *out, const T *in, const float *__restrict__ freqs, long total, int row,
                            int heads_per_row, int nrot, int HS, int pos0) {
    long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= total) return;
    const int half = HS / 2;
    const int d = (int)(idx % half);
    long t = idx / half;
    const int h = (int)(t % nrot);
    t /= nrot;  // flat row index b * row + r
    const int r = (int)(t % row);
    const float *f = freqs + (long)(pos0 + r) * HS + 2 * d;
    const float c = f[0], s = f[1];
    const long base = t * heads_per_row * HS + (long)h * HS + 2 * d;
    const float xr = to_float(in[base]), xi = to_float(in[base + 1]);
    out[base] = from_float<T>(xr * c - xi * s);
    out[base + 1] = from_float<T>(xr * s + xi * c);
}

template <typename T>
void rope(T *out, const T *in, const float *freqs, int batch, int row, int heads_per_row, int nrot, int HS, int pos0,
          cudaStream_t s) {
    long total = (long)batch * row * nrot * (HS / 2);
    if (total <= 0) return;
    if (out != in) {
        // heads beyond `nrot` (V) are copied unchanged
        WK_CHECK(cudaMemcpyAsync(out, in, sizeof(T) * (size_t)batch * row * heads_per_row * HS,
                                 cudaMemcpyDeviceToDevice, s));
    }
    rope_kernel<T><<<(unsigned)((total + 255) / 256), 256, 0, s>>>(out, out == in ? in : out, freqs, total, row,
                                                                  heads_per_row, nrot, HS, pos0);
    WK_CHECK_LAUNCH();
}
template void rope<float>(float *, const float *, const float *, int, int, int, int, int, int, cudaStream_t);
template void rope<__half>(__half *, const __half *, const float *, int, int, int, int, int, int, cudaStream_t);
template void rope<__nv_bfloat16>(__nv_bfloat16 *, const __nv_bfloat16 *, const float *, int, int, int, int, int, int,
                                  cudaStream_t);

// ------------------------------------------------------------ swiglu
// cuda.cu:176-205: out[r, c] = up * (gate * sigmoid(gate)), row = [up | gate].
template <typename T>
__global__ void swiglu_kernel(T *__restrict__ out, const T *__restrict__ in, long total, int C) {
    long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= total) return;
    const long r = idx / C;
    const int c = (int)(idx % C);
    const float u = to_float(in[r * 2 * C + c]);
    const float g = to_float(in[r * 2 * C + C + c]);
    const float sig = 1.0f / (1.0f + expf(-g));
    out[idx] = from_float<T>((g * sig) * u);
}

template <typename T> void swiglu(T *out, const T *in, long rows, int C, cudaStream_t s) {
    long total = rows * C;
    if (total <= 0) return;
    T *dst = out;
    // the reference runs this in place (cuda.cu:939), where output row r overlaps
    // input row r/2; write to scratch first when the ranges overlap
    const char *ib = (const char *)in, *ie = ib + sizeof(T) * total * 2;
    const char *ob = (const char *)out, *oe = ob + sizeof(T) * total;
    bool overlap = ob < ie && ib < oe;
    if (overlap) dst = (T *)scratch(sizeof(T) * total);
    swiglu_kernel<T><<<(unsigned)((total + 255) / 256), 256, 0, s>>>(dst, in, total, C);
    WK_CHECK_LAUNCH();
    if (overlap) WK_CHECK(cudaMemcpyAsync(out, dst, sizeof(T) * total, cudaMemcpyDeviceToDevice, s));
}
template void swiglu<float>(float *, const float *, long, int, cudaStream_t);
template void swiglu<__half>(__half *, const __half *, long, int, cudaStream_t);
template void swiglu<__nv_bfloat16>(__nv_bfloat16 *, const __nv_bfloat16 *, long, int, cudaStream_t);

// ------------------------------------------------------------ add / div
template <typename T> __global__ void add_kernel(T *out, const T *a, const T *b, long n) {
    long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = from_float<T>(to_float(a[i]) + to_float(b[i]));
}
template <typename T> void add(T *out, const T *a, const T *b, long n, cudaStream_t s) {
    if (n <= 0) return;
    add_kernel<T><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(out, a, b, n);
    WK_CHECK_LAUNCH();
}
template void add<float>(float *, const float *, const float *, long, cudaStream_t);
template void add<__half>(__half *, const __half *, const __half *, long, cudaStream_t);
template void add<__nv_bfloat16>(__nv_bfloat16 *, const __nv_bfloat16 *, const __nv_bfloat16 *, long, cudaStream_t);

__global__ void div_kernel(float *out, const float *a, const float *b, long n) {
    long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = a[i] / b[i];
}

// ------------------------------------------------------------ softmax (fp32)
// cuda.cu:86-158: row softmax.
__global__ void __launch_bounds__(256) softmax_kernel(float *out, const float *in, int col) {
    __shared__ float red[32];
    const float *x = in + (size_t)blockIdx.x * col;
    float *o = out + (size_t)blockIdx.x * col;
    float m = -INFINITY;
    for (int i = threadIdx.x; i < col; i += blockDim.x) m = fmaxf(m, x[i]);
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : -INFINITY;
        v = warp_max(v);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    m = red[0];
    __syncthreads();
    float sum = 0.f;
    for (int i = threadIdx.x; i < col; i += blockDim.x) {
        float e = expf(x[i] - m);
        o[i] = e;
        sum += e;
    }
    sum = warp_sum(sum);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        v = warp_sum(v);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float inv = 1.0f / red[0];
    for (int i = threadIdx.x; i < col; i += blockDim.x) o[i] *= inv;
}

// ------------------------------------------------------------ get_row
template <typename T>
__global__ void get_row_kernel(T *__restrict__ out, const T *__restrict__ in, int row, int col, int idx) {
    const int b = blockIdx.x;
    const T *src = in + ((size_t)b * row + idx) * col;
    for (int i = threadIdx.x; i < col; i += blockDim.x) out[(size_t)b * col + i] = src[i];
}
template <typename T> void get_row(T *out, const T *in, int batch, int row, int col, int idx, cudaStream_t s) {
    if (batch <= 0) return;
    if (idx < 0) idx += row;
    if (idx < 0 || idx >= row) WK_PANIC("row index %d out of range [0, %d)", idx, row);
    T *dst = out;
    bool overlap = (const void *)out < (const void *)(in + (size_t)batch * row * col) &&
                   (const void *)in < (const void *)(out + (size_t)batch * col);
    if (overlap) dst = (T *)scratch(sizeof(T) * (size_t)batch * col);
    get_row_kernel<T><<<batch, 256, 0, s>>>(dst, in, row, col, idx);
    WK_CHECK_LAUNCH();
    if (overlap) WK_CHECK(cudaMemcpyAsync(out, dst, sizeof(T) * (size_t)batch * col, cudaMemcpyDeviceToDevice, s));
}
template void get_row<float>(float *, const float *, int, int, int, int, cudaStream_t);
template void get_row<__half>(__half *, const __half *, int, int, int, int, cudaStream_t);
template void get_row<__nv_bfloat16>(__nv_bfloat16 *, const __nv_bfloat16 *, int, int, int, int, cudaStream_t);

// ------------------------------------------------------------ argmax
// cuda.cu:480-531.  The reference scans with 256 threads, thread tid owning the
// 16-byte packs tid, tid+256, ... (pack = 16 / sizeof(T) elements), keeps the
// first maximum it meets, and merges with a shfl_down tree that on ties keeps
// the lane (then the warp) with the smaller bit-reversed index.  argmax_key()
// encodes that order so that any reduction shape reproduces its choice.
__device__ __forceinline__ uint64_t argmax_key(long idx, int pack) {
    const long p = idx / pack;
    const uint32_t tid = (uint32_t)(p & 255), j = (uint32_t)(p >> 8), e = (uint32_t)(idx - p * pack);
    const uint32_t bw = __brev(tid >> 5) >> 27, bl = __brev(tid & 31) >> 27;
    return ((uint64_t)bw << 58) | ((uint64_t)bl << 53) | ((uint64_t)j << 8) | e;
}

__device__ __forceinline__ void argmax_merge(float &v, uint64_t &k, float ov, uint64_t ok) {
    if (ov > v || (ov == v && ok < k)) {
        v = ov;
        k = ok;
    }
}

template <typename T>
__global__ void __launch_bounds__(256) argmax_kernel(int *__restrict__ out, const T *__restrict__ in, int col) {
    __shared__ float sv[8];
    __shared__ uint64_t sk[8];
    constexpr int pack = 16 / sizeof(T);
    const T *x = in + (size_t)blockIdx.x * col;
    float best = -INFINITY;
    uint64_t bkey = ~0ull;
    const long n = (long)(col / pack) * pack;
    for (long i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = to_float(x[i]);
        if (v > best || (v == best && bkey != ~0ull)) {
            const uint64_t k = argmax_key(i, pack);
            if (v > best || k < bkey) {
                best = v;
                bkey = k;
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float ov = __shfl_xor_sync(0xffffffffu, best, o);
        uint64_t ok = __shfl_xor_sync(0xffffffffu, bkey, o);
        argmax_merge(best, bkey, ov, ok);
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = best;
        sk[threadIdx.x >> 5] = bkey;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; ++w) argmax_merge(best, bkey, sv[w], sk[w]);
        int idx = -1;
        if (bkey != ~0ull) {
            // decode the key back to the element index
            const uint32_t bw = (uint32_t)(bkey >> 58) & 31, bl = (uint32_t)(bkey >> 53) & 31;
            const uint32_t tid = ((__brev(bw) >> 27) << 5) | (__brev(bl) >> 27);
            const long j = (long)((bkey >> 8) & ((1ull << 45) - 1));
            const int e = (int)(bkey & 255);
            idx = (int)(((j << 8) + tid) * pack + e);
        }
        out[blockIdx.x] = idx;
    }
}

template <typename T> void argmax(int *out, const T *in, int rows, int col, cudaStream_t s) {
    if (rows <= 0) return;
    argmax_kernel<T><<<rows, 256, 0, s>>>(out, in, col);
    WK_CHECK_LAUNCH();
}
template void argmax<float>(int *, const float *, int, int, cudaStream_t);
template void argmax<__half>(int *, const __half *, int, int, cudaStream_t);
template void argmax<__nv_bfloat16>(int *, const __nv_bfloat16 *, int, int, cudaStream_t);

// ------------------------------------------------------------ repeat_qkv
// cuda.cu:437-467: [B, N, (NH + 2 kvNH) HS] -> [B, N, 3 NH HS], K/V repeated per group.
template <typename T>
__global__ void repeat_qkv_kernel(T *__restrict__ out, const T *__restrict__ in, long total, int NH, int kvNH, int HS) {
    long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= total) return;
    const int d = (int)(idx % HS);
    long t = idx / HS;
    const int h = (int)(t % NH);
    t /= NH;
    const int c = (int)(t % 3);
    const long row = t / 3;
    const int group = NH / kvNH;
    const long base = row * (long)(NH + 2 * kvNH) * HS;
    long src;
    if (c == 0)
        src = base + (long)h * HS + d;
    else if (c == 1)
        src = base + (long)NH * HS + (long)(h / group) * HS + d;
    else
        src = base + (long)(NH + kvNH) * HS + (long)(h / group) * HS + d;
    out[idx] = in[src];
}

}  // namespace wk

using namespace wk;

extern "C" {

// cuda.cu:1305-1308 (fp32 output)
void cuda_dequantize(void *out, const void *inp, int row, int col, int type) {
    ensure_init();
    if (type < 0 || type >= kDTypeCount) WK_PANIC("Unsupported quantization type: %d", type);
    if (type != kQ8_0 && type != kQ4_0) WK_PANIC("Unsupported quantization type: %s", kDTypes[type].name);
    if (col % kQ8Block) WK_PANIC("column count %d is not a multiple of %d", col, kQ8Block);
    if (type == kQ4_0)
        dequant_q4_0<float>((float *)out, inp, (long)row * (col / 32), stream());
    else
        dequant_q8_0<float>((float *)out, inp, (long)row * (col / kQ8Block), stream());
}

// cuda.cu:1232-1255
void cuda_embedding(void *out, const void *inp, const void *embd, int batch, int row, int col, int dtype) {
    ensure_init();
    if (dtype < 0 || dtype >= kDTypeCount) WK_PANIC("Unsupported quantization type: %d", dtype);
    if (dtype != kF32 && dtype != kF16 && dtype != kBF16 && dtype != kQ8_0 && dtype != kQ4_0)
        WK_PANIC("Unsupported embedding type: %s", kDTypes[dtype].name);
    if (col % kDTypes[dtype].block_size) WK_PANIC("column count %d is not a multiple of the block size", col);
    prefix_cache_embedding(out, (const int *)inp, embd, batch, row, col, dtype);
}

// cuda.cu:1156-1159 (fp32)
void cuda_rmsnorm(void *out, const void *inp, const void *weight, int row, int col, float eps) {
    ensure_init();
    rmsnorm<float>((float *)out, (const float *)inp, (const float *)weight, row, col, eps, stream());
}

// cuda.cu:1164-1167 (fp32)
void cuda_swiglu(void *out, const void *inp, int batch, int row, int col) {
    ensure_init();
    swiglu<float>((float *)out, (const float *)inp, (long)batch * row, col, stream());
}

// cuda.cu:1217-1220 (fp32)
void cuda_rope_qkv(void *out, const void *inp, const void *freqs, int batch, int row, int NH, int kvNH, int HS) {
    ensure_init();
    rope<float>((float *)out, (const float *)inp, (const float *)freqs, batch, row, NH + 2 * kvNH, NH + kvNH, HS, 0,
                stream());
}

// cuda.h:15 declares cuda_rope; the reference never defines it.  Same rotation
// on a [batch, row, NH, HS] fp32 tensor with freqs [row, HS].
void cuda_rope(void *out, const void *inp, const void *freqs, int batch, int row, int NH, int HS) {
    ensure_init();
    rope<float>((float *)out, (const float *)inp, (const float *)freqs, batch, row, NH, NH, HS, 0, stream());
}

// cuda.cu:1286-1293
void cuda_div(void *out, const void *a, const void *b, int row, int col) {
    ensure_init();
    long n = (long)row * col;
    if (n <= 0) return;
    div_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream()>>>((float *)out, (const float *)a, (const float *)b, n);
    WK_CHECK_LAUNCH();
}

// cuda.cu:1319-1322 (fp32)
void cuda_add(void *out, const void *a, const void *b, int row, int col) {
    ensure_init();
    add<float>((float *)out, (const float *)a, (const float *)b, (long)row * col, stream());
}

// cuda.cu:1120-1126
void cuda_softmax(void *output, void *input, int row, int col) {
    ensure_init();
    if (row <= 0) return;
    softmax_kernel<<<row, 256, 0, stream()>>>((float *)output, (const float *)input, col);
    WK_CHECK_LAUNCH();
}

// cuda.cu:1351-1354 (fp32)
void cuda_repeat_qkv(void *out, const void *inp, int batch, int row, int qNH, int kvNH, int HS) {
    ensure_init();
    if (kvNH <= 0 || qNH % kvNH) WK_PANIC("qNH (%d) must be a multiple of kvNH (%d)", qNH, kvNH);
    long total = (long)batch * row * 3 * qNH * HS;
    if (total <= 0) return;
    repeat_qkv_kernel<float><<<(unsigned)((total + 255) / 256), 256, 0, stream()>>>(
        (float *)out, (const float *)inp, total, qNH, kvNH, HS);
    WK_CHECK_LAUNCH();
}

// cuda.cu:1366-1369 (fp32)
void cuda_get_row(void *out, const void *inp, int batch, int row, int col, int idx) {
    ensure_init();
    get_row<float>((float *)out, (const float *)inp, batch, row, col, idx, stream());
}

// cuda.cu:1379-1382 (fp32)
void cuda_argmax(void *out, const void *inp, int row, int col) {
    ensure_init();
    argmax<float>((int *)out, (const float *)inp, row, col, stream());
}

}  // extern "C"
