// Dequant-fused GEMV for decode: out[m, n] = sum_k W[n, k] * X[m, k], M <= 8.
//
// Reference semantics (cuda.cu:1095-1111 + :270-341): quantised weights are
// dequantised to half, w = (half)(float(scale) * q), then multiplied with half
// activations with fp32 accumulation and one rounding to T at the store.
//
// Design (B200):
//  * A CTA of 4 warps owns 16-row weight tiles (grid-stride).  Each warp streams
//    its share of the tile's K-chunks (256 Q8_0 values = 272 B per row, or 128
//    16-bit values = 256 B per row) with 1-D bulk copies (cp.async.bulk, one per
//    row, 16 lanes in parallel) into a private 4-stage shared-memory ring
//    guarded by mbarriers.  The first stages are requested before
//    griddepcontrol.wait, so weight streaming overlaps the tail of the
//    producing kernel under programmatic dependent launch.
//  * Dequantisation happens in registers: four int8 quants become two exact
//    half2 by a byte-permute/subtract, then one half2 multiply by the block
//    scale gives exactly the reference's rounded fp16 weights.
//  * The inner product runs on mma.sync m16n8k16 (fp16 x fp16 products are exact
//    in fp32, accumulation in fp32 -- the reference's cuBLAS math); the 8 MMA
//    columns carry up to 8 activation rows at no extra cost.  The k index is
//    permuted within each 16-slice so that every lane consumes 4 consecutive
//    quant bytes per row (one 32-bit word).
//  * Per-warp partial tiles are reduced through shared memory and a fused
//    epilogue stores, adds the residual, applies RoPE and appends K/V to the
//    paged cache, applies SwiGLU, or reduces logits to an argmax.
//  * An optional RMSNorm prologue normalises X while staging it in shared memory.
#include "common.cuh"
#include "wukong_internal.cuh"

namespace wk {

namespace {

constexpr int kWarps = 4;
constexpr int kStages = 4;
constexpr int kTileRows = 16;
constexpr int kRowBytesMax = 272;  // per-row bytes of one stage (Q8_0: 8 blocks)

template <int WT> struct WFmt;
template <> struct WFmt<kQ8_0> {
    static constexpr int kChunk = 256;          // elements per row per stage
    static constexpr int kChunkBytes = 272;     // 8 blocks * 34
    static __host__ __device__ long row_bytes(int K) { return (long)(K / 32) * 34; }
    static __host__ __device__ int chunk_bytes(int elems) { return elems / 32 * 34; }
};
template <> struct WFmt<kF16> {
    static constexpr int kChunk = 128;
    static constexpr int kChunkBytes = 256;
    static __host__ __device__ long row_bytes(int K) { return (long)K * 2; }
    static __host__ __device__ int chunk_bytes(int elems) { return elems * 2; }
};
template <> struct WFmt<kBF16> : WFmt<kF16> {};

struct Smem {
    uint8_t *ring;   // [kWarps][kStages][16][kRowBytesMax]
    uint64_t *bars;  // [kWarps][kStages]
    uint2 *xs;       // [Kpad/16][M][4] x 4 values (8 bytes)
    float *red;      // [kWarps][16][8]
    float *misc;     // norm scales [8], logits partials
};

__device__ __forceinline__ int tile_row(const GemvArgs &a, int tile, int r) {
    if (a.epi == EPI_SWIGLU) return r < 8 ? tile * 8 + r : a.F + tile * 8 + (r - 8);
    return tile * kTileRows + r;
}
__device__ __forceinline__ int num_tiles(const GemvArgs &a) {
    return a.epi == EPI_SWIGLU ? (a.F + 7) / 8 : (a.N + kTileRows - 1) / kTileRows;
}
__device__ __forceinline__ bool row_valid(const GemvArgs &a, int tile, int r) {
    if (a.epi == EPI_SWIGLU) return tile * 8 + (r & 7) < a.F;
    return tile * kTileRows + r < a.N;
}

// Request the bytes of one (tile, chunk) unit into ring slot `slot` of warp `w`.
template <int WT>
__device__ __forceinline__ void issue_unit(const GemvArgs &a, const Smem &sm, int w, int slot, int tile, int chunk,
                                           int lane, bool bulk) {
    using F = WFmt<WT>;
    const long rb = F::row_bytes(a.K);
    const int e0 = chunk * F::kChunk;
    const int elems = min(F::kChunk, a.K - e0);
    const int bytes = F::chunk_bytes(elems);
    uint8_t *dst0 = sm.ring + ((size_t)(w * kStages + slot) * kTileRows) * kRowBytesMax;
    uint64_t *bar = sm.bars + w * kStages + slot;
    if (bulk) {
        int nvalid = 0;
#pragma unroll 4
        for (int r = 0; r < kTileRows; ++r) nvalid += row_valid(a, tile, r) ? 1 : 0;
        if (lane == 0) mbar_expect_tx(bar, (uint32_t)(nvalid * bytes));
        __syncwarp();
        if (lane < kTileRows && row_valid(a, tile, lane)) {
            const uint8_t *src = a.w + (long)tile_row(a, tile, lane) * rb + F::chunk_bytes(e0);
            bulk_g2s(dst0 + lane * kRowBytesMax, src, (uint32_t)bytes, bar);
        }
    } else {
        // unaligned rows: synchronous copy by the warp, zero padding to a 16-slice
        const int padded = F::chunk_bytes(((elems + 15) / 16) * 16);
        for (int r = 0; r < kTileRows; ++r) {
            const bool ok = row_valid(a, tile, r);
            const uint8_t *src = ok ? a.w + (long)tile_row(a, tile, r) * rb + F::chunk_bytes(e0) : nullptr;
            for (int i = lane; i < padded; i += 32) dst0[r * kRowBytesMax + i] = (ok && i < bytes) ? src[i] : 0;
        }
        __syncwarp();
    }
}

// Consume one unit: accumulate the 16 x 8 tile over the chunk's k-slices.
template <int WT>
__device__ __forceinline__ void consume_unit(const GemvArgs &a, const Smem &sm, int w, int slot, int chunk, int lane,
                                             float (&c)[4]) {
    using F = WFmt<WT>;
    const int g = lane >> 2, t = lane & 3;
    const int e0 = chunk * F::kChunk;
    const int elems = min(F::kChunk, a.K - e0);
    const uint8_t *st = sm.ring + ((size_t)(w * kStages + slot) * kTileRows) * kRowBytesMax;
    const uint8_t *r0 = st + g * kRowBytesMax;
    const uint8_t *r1 = st + (g + 8) * kRowBytesMax;
    const int M = a.M;
    const int s_base = e0 / 16;
    if constexpr (WT == kQ8_0) {
        const int nblk = elems / 32;
#pragma unroll 2
        for (int b = 0; b < nblk; ++b) {
            const int off = b * 34;
            const __half2 s0 = __half2half2(*reinterpret_cast<const __half *>(r0 + off));
            const __half2 s1 = __half2half2(*reinterpret_cast<const __half *>(r1 + off));
            uint32_t q0[2], q1[2];  // [slice] quant words for rows g, g+8
            if (b & 1) {
                // quants start 4-byte aligned (34 * odd + 2 = 0 mod 4)
                q0[0] = *reinterpret_cast<const uint32_t *>(r0 + off + 2 + 4 * t);
                q0[1] = *reinterpret_cast<const uint32_t *>(r0 + off + 18 + 4 * t);
                q1[0] = *reinterpret_cast<const uint32_t *>(r1 + off + 2 + 4 * t);
                q1[1] = *reinterpret_cast<const uint32_t *>(r1 + off + 18 + 4 * t);
            } else {
                const uint32_t *p0 = reinterpret_cast<const uint32_t *>(r0 + off + 4 * t);
                const uint32_t *p1 = reinterpret_cast<const uint32_t *>(r1 + off + 4 * t);
                q0[0] = __byte_perm(p0[0], p0[1], 0x5432);
                q0[1] = __byte_perm(p0[4], p0[5], 0x5432);
                q1[0] = __byte_perm(p1[0], p1[1], 0x5432);
                q1[1] = __byte_perm(p1[4], p1[5], 0x5432);
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                __half2 lo0, hi0, lo1, hi1;
                i8x4_to_h2x2(q0[h], lo0, hi0);
                i8x4_to_h2x2(q1[h], lo1, hi1);
                const uint32_t a0 = h2_as_u32(__hmul2(lo0, s0)), a2 = h2_as_u32(__hmul2(hi0, s0));
                const uint32_t a1 = h2_as_u32(__hmul2(lo1, s1)), a3 = h2_as_u32(__hmul2(hi1, s1));
                uint32_t b0 = 0, b1 = 0;
                if (g < M) {
                    const uint2 xv = sm.xs[((s_base + 2 * b + h) * M + g) * 4 + t];
                    b0 = xv.x;
                    b1 = xv.y;
                }
                mma_f16(c, a0, a1, a2, a3, b0, b1);
            }
        }
    } else {
        const int ns = (elems + 15) / 16;
#pragma unroll 4
        for (int s = 0; s < ns; ++s) {
            const uint2 w0 = *reinterpret_cast<const uint2 *>(r0 + s * 32 + 8 * t);
            const uint2 w1 = *reinterpret_cast<const uint2 *>(r1 + s * 32 + 8 * t);
            uint32_t b0 = 0, b1 = 0;
            if (g < M) {
                const uint2 xv = sm.xs[((s_base + s) * M + g) * 4 + t];
                b0 = xv.x;
                b1 = xv.y;
            }
            if constexpr (WT == kBF16)
                mma_bf16(c, w0.x, w1.x, w0.y, w1.y, b0, b1);
            else
                mma_f16(c, w0.x, w1.x, w0.y, w1.y, b0, b1);
        }
    }
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    T ha = from_float<T>(a), hb = from_float<T>(b);
    return (uint32_t)*reinterpret_cast<uint16_t *>(&ha) | ((uint32_t)*reinterpret_cast<uint16_t *>(&hb) << 16);
}

// Stage X (optionally RMS-normalised, rounded to T as the reference stores its
// rmsnorm output) into the permuted fragment layout.
template <typename T>
__device__ void stage_x(const GemvArgs &a, const Smem &sm, int Kpad) {
    const int M = a.M;
    const T *x = reinterpret_cast<const T *>(a.x);
    if (a.norm_w) {
        // one warp per activation row: sum of squares
        const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
        for (int m = wid; m < M; m += kWarps) {
            const T *xr = x + (long)m * a.ldx;
            float ss = 0.f;
            for (int k = lane; k < a.K; k += 32) {
                float v = to_float(xr[k]);
                ss += v * v;
            }
            ss = warp_sum(ss);
            if (lane == 0) sm.misc[m] = rsqrtf(ss / (float)a.K + a.eps);
        }
        __syncthreads();
    }
    const int nq = Kpad / 4;
    for (int i = threadIdx.x; i < nq * M; i += blockDim.x) {
        const int m = i % M, kq = i / M;
        const int k = kq * 4;
        const T *xr = x + (long)m * a.ldx;
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float xv = (k + j < a.K) ? to_float(xr[k + j]) : 0.f;
            if (a.norm_w && k + j < a.K) xv = (xv * sm.misc[m]) * a.norm_w[k + j];
            v[j] = xv;
        }
        uint2 pk;
        pk.x = pack2<T>(v[0], v[1]);
        pk.y = pack2<T>(v[2], v[3]);
        sm.xs[((kq >> 2) * M + m) * 4 + (kq & 3)] = pk;
    }
}

__device__ __forceinline__ uint64_t logits_key(long idx, int pack) {
    const long p = idx / pack;
    const uint32_t tid = (uint32_t)(p & 255), j = (uint32_t)(p >> 8), e = (uint32_t)(idx - p * pack);
    const uint32_t bw = __brev(tid >> 5) >> 27, bl = __brev(tid & 31) >> 27;
    return ((uint64_t)bw << 58) | ((uint64_t)bl << 53) | ((uint64_t)j << 8) | e;
}

template <typename T>
__device__ void epilogue(const GemvArgs &a, const Smem &sm, int tile, float (&best_v)[8], uint64_t (&best_k)[8]) {
    // sum the warps' partial tiles: tid -> (row r, column m)
    const int tid = threadIdx.x;
    const int r = tid >> 3, m = tid & 7;
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) acc += sm.red[(w * 16 + r) * 8 + m];
    __syncthreads();
    sm.red[r * 8 + m] = acc;  // reduced tile in slot of warp 0
    __syncthreads();
    if (m >= a.M || !row_valid(a, tile, r)) return;
    const int n = tile_row(a, tile, r);
    switch (a.epi) {
    case EPI_STORE: {
        if (a.bias) acc += to_float(reinterpret_cast<const T *>(a.bias)[n]);
        reinterpret_cast<T *>(a.out)[(long)m * a.ldo + n] = from_float<T>(acc);
        break;
    }
    case EPI_RESID: {
        const float y = round_to<T>(acc);
        const float rv = to_float(reinterpret_cast<const T *>(a.res)[(long)m * a.ldr + n]);
        reinterpret_cast<T *>(a.out)[(long)m * a.ldo + n] = from_float<T>(rv + y);
        break;
    }
    case EPI_QKV: {
        const float y = round_to<T>(acc);
        const int pos = a.pos[m];
        if (n < a.nq + a.nk) {
            const float yp = round_to<T>(sm.red[(r ^ 1) * 8 + m]);
            const int dd = (n - (n < a.nq ? 0 : a.nq)) % a.hd;
            const float *f = a.freqs + (long)pos * a.hd + (dd & ~1);
            const float cs = f[0], sn = f[1];
            const float o = (n & 1) ? (yp * sn + y * cs) : (y * cs - yp * sn);
            if (n < a.nq) {
                reinterpret_cast<T *>(a.out)[(long)m * a.ldo + n] = from_float<T>(o);
            } else {
                const int kh = (n - a.nq) / a.hd;
                const long page = a.block_table[(long)a.seq[m] * a.max_pages + pos / a.page];
                const long off = ((page * a.kv_heads + kh) * a.page + pos % a.page) * a.hd + dd;
                reinterpret_cast<T *>(a.kpool)[off] = from_float<T>(o);
            }
        } else {
            const int dd = (n - a.nq - a.nk) % a.hd, vh = (n - a.nq - a.nk) / a.hd;
            const long page = a.block_table[(long)a.seq[m] * a.max_pages + pos / a.page];
            const long off = ((page * a.kv_heads + vh) * a.page + pos % a.page) * a.hd + dd;
            reinterpret_cast<T *>(a.vpool)[off] = from_float<T>(y);
        }
        break;
    }
    case EPI_SWIGLU: {
        if (r < 8) {
            const float u = round_to<T>(acc);
            const float gt = round_to<T>(sm.red[(r + 8) * 8 + m]);
            const float sig = 1.0f / (1.0f + expf(-gt));
            reinterpret_cast<T *>(a.out)[(long)m * a.ldo + tile * 8 + r] = from_float<T>((gt * sig) * u);
        }
        break;
    }
    case EPI_LOGITS: {
        const float y = round_to<T>(acc);
        if (a.out) reinterpret_cast<T *>(a.out)[(long)m * a.ldo + n] = from_float<T>(y);
        const long lim = (long)(a.N / a.pack) * a.pack;
        if (n < lim && (y > best_v[m] || (y == best_v[m] && best_k[m] != ~0ull))) {
            const uint64_t k = logits_key(n, a.pack);
            if (y > best_v[m] || k < best_k[m]) {
                best_v[m] = y;
                best_k[m] = k;
            }
        }
        break;
    }
    }
}

template <typename T, int WT>
__global__ void __launch_bounds__(kWarps * 32) gemv_kernel(const GemvArgs a) {
    using F = WFmt<WT>;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const int nchunks = (a.K + F::kChunk - 1) / F::kChunk;
    const int Kpad = nchunks * F::kChunk;
    Smem sm;
    sm.ring = smem_raw;
    sm.bars = reinterpret_cast<uint64_t *>(sm.ring + (size_t)kWarps * kStages * kTileRows * kRowBytesMax);
    sm.xs = reinterpret_cast<uint2 *>(sm.bars + kWarps * kStages);
    sm.red = reinterpret_cast<float *>(sm.xs + (size_t)(Kpad / 4) * a.M);
    sm.misc = sm.red + kWarps * 16 * 8;

    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = num_tiles(a);
    const bool bulk = a.bulk != 0;
    if (threadIdx.x < kWarps * kStages) mbar_init(sm.bars + threadIdx.x, 1);
    mbar_fence_init();
    __syncthreads();

    // this warp's unit sequence: tiles blockIdx.x, +gridDim.x, ...; chunks w, w+4, ...
    int p_tile = blockIdx.x, p_chunk = w;  // producer cursor
    auto advance = [&](int &tile, int &chunk) {
        chunk += kWarps;
        if (chunk >= nchunks) {
            chunk = w;
            tile += gridDim.x;
        }
    };
    // a warp with no chunk in this K (w >= nchunks) idles in the k-loop
    const bool has_work = w < nchunks;
    int issued = 0;
    if (bulk && has_work) {
        for (; issued < kStages && p_tile < ntiles; ++issued) {
            issue_unit<WT>(a, sm, w, issued % kStages, p_tile, p_chunk, lane, true);
            advance(p_tile, p_chunk);
        }
    }
    // weights are ready to stream; wait for the producer of X, then let the next
    // kernel in the stream start its own weight prefetch
    pdl_wait();
    pdl_trigger();
    stage_x<T>(a, sm, Kpad);
    __syncthreads();

    float best_v[8];
    uint64_t best_k[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        best_v[m] = -INFINITY;
        best_k[m] = ~0ull;
    }

    int consumed = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        float c[4] = {0.f, 0.f, 0.f, 0.f};
        if (has_work) {
            for (int chunk = w; chunk < nchunks; chunk += kWarps) {
                const int slot = consumed % kStages;
                bool ready = true;
                if (bulk) {
                    // a copy that never lands is reported, not waited on forever
                    ready = mbar_wait_bounded(sm.bars + w * kStages + slot, (consumed / kStages) & 1, a.err, 1);
                } else {
                    issue_unit<WT>(a, sm, w, slot, tile, chunk, lane, false);
                }
                if (ready) consume_unit<WT>(a, sm, w, slot, chunk, lane, c);
                __syncwarp();
                ++consumed;
                if (bulk && p_tile < ntiles) {
                    // refill the slot just consumed
                    issue_unit<WT>(a, sm, w, (issued) % kStages, p_tile, p_chunk, lane, true);
                    ++issued;
                    advance(p_tile, p_chunk);
                }
            }
        }
        // partial tile of this warp -> shared memory (rows g, g+8; columns 2t, 2t+1)
        const int g = lane >> 2, t = lane & 3;
        float *red = sm.red + w * 16 * 8;
        red[g * 8 + 2 * t] = c[0];
        red[g * 8 + 2 * t + 1] = c[1];
        red[(g + 8) * 8 + 2 * t] = c[2];
        red[(g + 8) * 8 + 2 * t + 1] = c[3];
        __syncthreads();
        epilogue<T>(a, sm, tile, best_v, best_k);
        __syncthreads();
    }

    if (a.epi == EPI_LOGITS) {
        // per-CTA argmax partials: reduce over the 16 row-threads of each column m
        const int tid = threadIdx.x, m = tid & 7;
        float v = best_v[m];
        uint64_t k = best_k[m];
        float *sv = sm.misc;  // [16][8]
        uint64_t *sk = reinterpret_cast<uint64_t *>(sm.misc + 128);
        sv[tid] = v;
        sk[tid] = k;
        __syncthreads();
        if (tid < 8 && tid < a.M) {
            for (int r = 1; r < 16; ++r) {
                const float ov = sv[r * 8 + tid];
                const uint64_t ok = sk[r * 8 + tid];
                if (ov > v || (ov == v && ok < k)) {
                    v = ov;
                    k = ok;
                }
            }
            a.part_val[(long)blockIdx.x * 8 + tid] = v;
            a.part_key[(long)blockIdx.x * 8 + tid] = k;
        }
        // the last CTA to finish reduces the partials to token ids
        __shared__ int last;
        __threadfence();
        __syncthreads();
        if (tid == 0) last = (atomicAdd(a.counter, 1) == (int)gridDim.x - 1);
        __syncthreads();
        if (last) {
            __threadfence();
            if (tid < a.M) {
                float bv = -INFINITY;
                uint64_t bk = ~0ull;
                for (int b = 0; b < (int)gridDim.x; ++b) {
                    const float ov = ((volatile float *)a.part_val)[(long)b * 8 + tid];
                    const uint64_t ok = ((volatile unsigned long long *)a.part_key)[(long)b * 8 + tid];
                    if (ov > bv || (ov == bv && ok < bk)) {
                        bv = ov;
                        bk = ok;
                    }
                }
                int idx = -1;
                if (bk != ~0ull) {
                    const uint32_t bw = (uint32_t)(bk >> 58) & 31, bl = (uint32_t)(bk >> 53) & 31;
                    const uint32_t tid8 = ((__brev(bw) >> 27) << 5) | (__brev(bl) >> 27);
                    const long j = (long)((bk >> 8) & ((1ull << 45) - 1));
                    idx = (int)(((j << 8) + tid8) * a.pack + (int)(bk & 255));
                }
                a.tokens[tid] = idx;
            }
            if (tid == 0) *a.counter = 0;
        }
    }
}

size_t gemv_smem_bytes(int K, int M, int wt) {
    const int chunk = wt == kQ8_0 ? WFmt<kQ8_0>::kChunk : WFmt<kF16>::kChunk;
    const int Kpad = (K + chunk - 1) / chunk * chunk;
    return (size_t)kWarps * kStages * kTileRows * kRowBytesMax + kWarps * kStages * 8 + (size_t)(Kpad / 4) * M * 8 +
           kWarps * 16 * 8 * 4 + 128 * 4 + 128 * 8;
}

template <typename T, int WT> void launch(const GemvArgs &a, int grid, size_t smem, cudaStream_t s, bool pdl) {
    auto kern = gemv_kernel<T, WT>;
    static bool configured[2] = {false, false};
    (void)configured;
    WK_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kWarps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    WK_CHECK(cudaLaunchKernelEx(&cfg, kern, a));
}

}  // namespace

bool gemv_supported(int wtype, int act, int K) {
    if (wtype == kQ8_0) return act == kF16 && K % 32 == 0;
    if (wtype == kF16) return act == kF16 && K % 16 == 0;
    if (wtype == kBF16) return act == kBF16 && K % 16 == 0;
    return false;
}

void gemv(GemvArgs a, int act, cudaStream_t s) {
    if (a.M <= 0 || a.M > 8) WK_PANIC("gemv: M=%d outside [1, 8]", a.M);
    if (!gemv_supported(a.wtype, act, a.K)) WK_PANIC("gemv: unsupported wtype %d / act %d / K %d", a.wtype, act, a.K);
    const int chunkb = a.wtype == kQ8_0 ? 272 : 256;
    const long rb = a.wtype == kQ8_0 ? (long)(a.K / 32) * 34 : (long)a.K * 2;
    (void)chunkb;
    a.bulk = ((uintptr_t)a.w % 16 == 0) && (rb % 16 == 0) ? 1 : 0;
    if (!a.err) a.err = g_rt.d_error;
    const size_t smem = gemv_smem_bytes(a.K, a.M, a.wtype);
    if ((int)smem > g_rt.max_smem_optin) WK_PANIC("gemv: K=%d M=%d needs %zu B of shared memory", a.K, a.M, smem);
    const int ntiles = a.epi == EPI_SWIGLU ? (a.F + 7) / 8 : (a.N + kTileRows - 1) / kTileRows;
    int per_sm = smem <= 100 * 1024 ? 2 : 1;
    int grid = ntiles < g_rt.num_sms * per_sm ? ntiles : g_rt.num_sms * per_sm;
    if (a.epi == EPI_LOGITS && grid > kMaxLogitCtas) grid = kMaxLogitCtas;
    const bool pdl = g_rt.pdl && a.pdl;
    if (a.wtype == kQ8_0)
        launch<__half, kQ8_0>(a, grid, smem, s, pdl);
    else if (a.wtype == kF16)
        launch<__half, kF16>(a, grid, smem, s, pdl);
    else
        launch<__nv_bfloat16, kBF16>(a, grid, smem, s, pdl);
}

}  // namespace wk
