// Dequant-fused GEMV for decode: out[m, n] = sum_k W[n, k] * X[m, k], M <= 8.
//
// Reference semantics (cuda.cu:1095-1111 + :270-341): quantised weights are
// dequantised to half, w = (half)(float(scale) * q), then multiplied with half
// activations with fp32 accumulation and one rounding to T at the store.
//
// Design (B200):
//  * A CTA of 8 warps owns 16-row weight tiles (grid-stride).  Each warp streams
//    its share of the tile's K-chunks (256 Q8_0 values = 272 B per row, or 128
//    16-bit values = 256 B per row) into a private 3-stage shared-memory ring
//    with 16-byte cp.async copies: every lane moves one 16-byte piece per
//    instruction, so each instruction is a fully coalesced 512-byte request.
//    The first stages are requested before griddepcontrol.wait, so weight
//    streaming overlaps the tail of the producing kernel under programmatic
//    dependent launch.
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
#include "timeline.cuh"
#include "wukong_internal.cuh"

namespace wk {

namespace {

constexpr int kWarps = 8;
constexpr int kStages = 3;
constexpr size_t kXStageMax = 32 * 1024;  // X is staged in shared memory up to this size
constexpr int kTileRows = 16;
constexpr int kStageBytes = kTileRows * 272;  // one unit: 16 rows x (8 Q8_0 blocks | 128 halves)

template <int WT> struct WFmt;
template <> struct WFmt<kQ8_0> {
    static constexpr int kChunk = 256;  // elements per row per stage
    static constexpr int kRowB = 272;   // bytes per row per stage (8 blocks)
    static __host__ __device__ long row_bytes(int K) { return (long)(K / 32) * 34; }
    static __host__ __device__ int chunk_bytes(int elems) { return elems / 32 * 34; }
};
template <> struct WFmt<kQ4_0> {
    static constexpr int kChunk = 256;  // elements per row per stage
    static constexpr int kRowB = 144;   // bytes per row per stage (8 blocks of 18)
    static __host__ __device__ long row_bytes(int K) { return (long)(K / 32) * 18; }
    static __host__ __device__ int chunk_bytes(int elems) { return elems / 32 * 18; }
};
template <> struct WFmt<kF16> {
    static constexpr int kChunk = 128;
    static constexpr int kRowB = 256;
    static __host__ __device__ long row_bytes(int K) { return (long)K * 2; }
    static __host__ __device__ int chunk_bytes(int elems) { return elems * 2; }
};
template <> struct WFmt<kBF16> : WFmt<kF16> {};

struct Smem {
    uint8_t *ring;    // [kWarps][kStages][16][kRowB]
    uint64_t *bars;   // [kWarps][kStages] TMA completion
    // X as the MMA B operand: row-major [M][ld] 16-bit values viewed as uint2.
    // Lane (g, t) of k-slice s reads the 4 values at k = 16 s + 4 t of row g,
    // i.e. uint2 (4 s + t), which matches the A-side k permutation.  Points to
    // global memory, or to shared memory when an RMSNorm prologue is fused.
    const uint2 *xsrc;
    long xld;       // row stride in uint2
    uint2 *xn;      // [M][Kpad / 4] normalised X (RMSNorm prologue only)
    float *red;     // [kWarps][16][8]
    float *misc;    // norm scales [8], logits partials [128] + keys [128]
};

// 2-D TMA tile load into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"((uint64_t)map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

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
// TMA path: lane 0 issues one 2-D box of 16 rows (two boxes of 8 rows for the
// up|gate pairing of SwiGLU); rows past N arrive zero-filled.  Otherwise (rows
// that are not 16-byte aligned) a synchronous copy by the warp, zero padded.
template <int WT>
__device__ __forceinline__ void issue_unit(const GemvArgs &a, const Smem &sm, int w, int slot, int tile, int chunk,
                                           int lane, bool tma, int ns) {
    using F = WFmt<WT>;
    const int e0 = chunk * F::kChunk;
    uint8_t *dst0 = sm.ring + (size_t)(w * ns + slot) * kStageBytes;
    if (tma) {
        if (lane == 0) {
            uint64_t *bar = sm.bars + w * ns + slot;
            mbar_expect_tx(bar, kTileRows * F::kRowB);
            const int x = F::chunk_bytes(e0) / 2;  // uint16 column of the box
            if (a.epi == EPI_SWIGLU) {
                tma_load_2d(dst0, &a.wmap, x, tile * 8, bar);
                tma_load_2d(dst0 + 8 * F::kRowB, &a.wmap, x, a.F + tile * 8, bar);
            } else {
                tma_load_2d(dst0, &a.wmap, x, tile * kTileRows, bar);
            }
        }
    } else {
        const long rb = F::row_bytes(a.K);
        const int elems = min(F::kChunk, a.K - e0);
        const int bytes = F::chunk_bytes(elems);
        const int padded = F::chunk_bytes(((elems + 15) / 16) * 16);
        for (int r = 0; r < kTileRows; ++r) {
            const bool ok = row_valid(a, tile, r);
            const uint8_t *src = ok ? a.w + (long)tile_row(a, tile, r) * rb + F::chunk_bytes(e0) : nullptr;
            for (int i = lane; i < padded; i += 32) dst0[r * F::kRowB + i] = (ok && i < bytes) ? src[i] : 0;
        }
    }
}

// Issue the next unit of this warp's sequence into `slot` and advance the
// cursor: chunks cstart, cstart + cstep, ... of tiles p_tile, p_tile + tstep, ...
template <int WT>
__device__ __forceinline__ void produce_unit(const GemvArgs &a, const Smem &sm, int w, int slot, int lane,
                                             bool has_work, int ntiles, int nchunks, int &p_tile, int &p_chunk,
                                             int cstart, int cstep, int tstep, int ns) {
    if (has_work && p_tile < ntiles) {
        issue_unit<WT>(a, sm, w, slot, p_tile, p_chunk, lane, true, ns);
        p_chunk += cstep;
        if (p_chunk >= nchunks) {
            p_chunk = cstart;
            p_tile += tstep;
        }
    }
}

// Consume one unit: accumulate the 16 x 8 tile over the chunk's k-slices into
// two independent accumulators (even / odd slice) to halve the MMA chain.
template <int WT>
__device__ __forceinline__ void consume_unit(const GemvArgs &a, const Smem &sm, int w, int slot, int chunk, int lane,
                                             float (&c)[2][4], int ns) {
    using F = WFmt<WT>;
    const int g = lane >> 2, t = lane & 3;
    const int e0 = chunk * F::kChunk;
    const int elems = min(F::kChunk, a.K - e0);
    const uint8_t *st = sm.ring + (size_t)(w * ns + slot) * kStageBytes;
    const uint8_t *r0 = st + g * F::kRowB;
    const uint8_t *r1 = st + (g + 8) * F::kRowB;
    const int M = a.M;
    const bool has_x = g < M;
    const uint2 *xl = sm.xsrc + (has_x ? g : 0) * sm.xld + (e0 / 16) * 4 + t;  // slice e0/16 of row g
    constexpr int xstep = 4;                                                   // uint2 per slice
    if constexpr (WT == kQ4_0) {
        const int nblk = elems / 32;
        if (nblk == 8) {
            uint2 xv[16];
#pragma unroll
            for (int s = 0; s < 16; ++s) {
                xv[s] = xl[s * xstep];
                if (!has_x) xv[s] = make_uint2(0u, 0u);
            }
#pragma unroll
            for (int b = 0; b < 8; ++b) q4_block(r0, r1, b * 18, (b & 1) != 0, t, xv[2 * b], xv[2 * b + 1], c);
        } else {
            for (int b = 0; b < nblk; ++b) {
                uint2 x0 = xl[(2 * b) * xstep], x1 = xl[(2 * b + 1) * xstep];
                if (!has_x) x0 = x1 = make_uint2(0u, 0u);
                q4_block(r0, r1, b * 18, (b & 1) != 0, t, x0, x1, c);
            }
        }
    } else if constexpr (WT == kQ8_0) {
        const int nblk = elems / 32;
        if (nblk == 8) {
            // full chunk: fetch the 16 B fragments first so their latency overlaps
            uint2 xv[16];
#pragma unroll
            for (int s = 0; s < 16; ++s) {
                xv[s] = xl[s * xstep];
                if (!has_x) xv[s] = make_uint2(0u, 0u);
            }
#pragma unroll
            for (int b = 0; b < 8; ++b) q8_block(r0, r1, b * 34, (b & 1) != 0, t, xv[2 * b], xv[2 * b + 1], c);
        } else {
            for (int b = 0; b < nblk; ++b) {
                uint2 x0 = xl[(2 * b) * xstep], x1 = xl[(2 * b + 1) * xstep];
                if (!has_x) x0 = x1 = make_uint2(0u, 0u);
                q8_block(r0, r1, b * 34, (b & 1) != 0, t, x0, x1, c);
            }
        }
    } else {
        const int ns = (elems + 15) / 16;
        // slices in pairs (a register array indexed by a runtime value would live in local memory)
#pragma unroll 2
        for (int s = 0; s < ns; s += 2) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                if (s + h < ns) {
                    const int sl = s + h;
                    const uint2 w0 = *reinterpret_cast<const uint2 *>(r0 + sl * 32 + 8 * t);
                    const uint2 w1 = *reinterpret_cast<const uint2 *>(r1 + sl * 32 + 8 * t);
                    uint2 xv = xl[sl * xstep];
                    if (!has_x) xv = make_uint2(0u, 0u);
                    if constexpr (WT == kBF16)
                        mma_bf16(c[h], w0.x, w1.x, w0.y, w1.y, xv.x, xv.y);
                    else
                        mma_f16(c[h], w0.x, w1.x, w0.y, w1.y, xv.x, xv.y);
                }
            }
        }
    }
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    T ha = from_float<T>(a), hb = from_float<T>(b);
    return (uint32_t)*reinterpret_cast<uint16_t *>(&ha) | ((uint32_t)*reinterpret_cast<uint16_t *>(&hb) << 16);
}

// RMSNorm weights held in registers from before griddepcontrol.wait (they do
// not depend on the previous kernel): thread t takes k = 4 (t + 256 j), j < 4,
// which covers K <= 4096; larger K loads the rest in the normalise loop (one
// L2 round trip per row and quad: at Llama-3.1-70B's K = 8192 and 4 rows about
// 11 us of prologue per normalising launch).  Eight register quads, or four
// more loaded beside the row copies, cover K = 8192 but cost the 1B decode
// step 4.4 % and the 8B step 1.6 % (registers held across the wait).
constexpr int kNormRegs = 4;
struct NormW {
    float4 v[kNormRegs];
};
__device__ __forceinline__ float4 load_norm4(const float *w, int k) {
    if ((reinterpret_cast<uintptr_t>(w) & 15) == 0) return *reinterpret_cast<const float4 *>(w + k);
    return make_float4(w[k], w[k + 1], w[k + 2], w[k + 3]);
}
__device__ __forceinline__ void norm_pre(const GemvArgs &a, NormW &nw) {
#pragma unroll
    for (int j = 0; j < kNormRegs; ++j) {
        const int k = (threadIdx.x + j * blockDim.x) * 4;
        nw.v[j] = k < a.K ? load_norm4(a.norm_w, k) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// RMSNorm prologue: normalise X, rounded to T as the reference stores its
// rmsnorm output (cuda.cu:533-601), into shared memory [M][Kpad] (zero padded).
// Sum-of-squares order (the persistent kernel follows it too): thread t adds
// the quads (4 consecutive values) k/4 = t, t + 256, ... of a row in that order,
// its warp sums the threads by butterfly, then the 8 warps' sums are added in
// warp order.  One row (decode) with K <= 4096 stays in registers from the load
// to the normalised store; more rows go through shared memory in the same order.
template <typename T>
__device__ __forceinline__ void quad_ss(uint2 q, float &ss) {
    const T *e = reinterpret_cast<const T *>(&q);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float f = to_float(e[j]);
        ss += f * f;
    }
}
template <typename T>
__device__ __forceinline__ uint2 quad_norm(uint2 q, float r, float4 w) {
    const T *e = reinterpret_cast<const T *>(&q);
    uint2 pk;
    pk.x = pack2<T>((to_float(e[0]) * r) * w.x, (to_float(e[1]) * r) * w.y);
    pk.y = pack2<T>((to_float(e[2]) * r) * w.z, (to_float(e[3]) * r) * w.w);
    return pk;
}
template <typename T>
__device__ void stage_xn(const GemvArgs &a, const Smem &sm, int Kpad, const NormW &nw) {
    const int M = a.M;
    const T *x = reinterpret_cast<const T *>(a.x);
    const int nq = Kpad / 4, total = nq * M, nt = blockDim.x, tid = threadIdx.x;
    const int wid = tid >> 5, lane = tid & 31;
    const int kq_end = a.K / 4;  // quads holding data (K is a multiple of 16)
    auto ld = [&](int i) -> uint2 {
        const int m = i / nq, k = (i - m * nq) * 4;
        return k < a.K ? *reinterpret_cast<const uint2 *>(x + (long)m * a.ldx + k) : make_uint2(0u, 0u);
    };
    float *wsum = sm.red;  // [8 warps][8 rows] (the tiles use sm.red only later)
    if (a.norm_w && M == 1 && nq <= kNormRegs * nt) {
        uint2 v[kNormRegs];
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < kNormRegs; ++j) {
            const int kq = tid + j * nt;
            v[j] = kq < nq ? ld(kq) : make_uint2(0u, 0u);
        }
#pragma unroll
        for (int j = 0; j < kNormRegs; ++j)
            if (tid + j * nt < kq_end) quad_ss<T>(v[j], ss);
        ss = warp_sum(ss);
        if (lane == 0) wsum[wid * 8] = ss;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) tot += wsum[w * 8];
        const float r = rsqrtf(tot / (float)a.K + a.eps);
#pragma unroll
        for (int j = 0; j < kNormRegs; ++j) {
            const int kq = tid + j * nt;
            if (kq < nq) sm.xn[kq] = kq < kq_end ? quad_norm<T>(v[j], r, nw.v[j]) : make_uint2(0u, 0u);
        }
        return;  // the caller's barrier publishes the rows
    }
    // every quad of every row in flight at once (8-byte asynchronous copies, then
    // one wait): several rows of a wide layer cost one L2 round trip, not one per
    // batch of loads a thread can hold in registers
    for (int i = tid; i < total; i += nt) {
        const int m = i / nq, k = (i - m * nq) * 4;
        if (k < a.K)
            asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(&sm.xn[i])),
                         "l"(x + (long)m * a.ldx + k)
                         : "memory");
        else
            sm.xn[i] = make_uint2(0u, 0u);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    if (!a.norm_w) return;
    for (int m = 0; m < M; ++m) {
        float ss = 0.f;
        for (int kq = tid; kq < kq_end; kq += nt) quad_ss<T>(sm.xn[m * nq + kq], ss);
        ss = warp_sum(ss);
        if (lane == 0) wsum[wid * 8 + m] = ss;
    }
    __syncthreads();
    for (int m = 0; m < M; ++m) {
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) tot += wsum[w * 8 + m];
        const float r = rsqrtf(tot / (float)a.K + a.eps);
#pragma unroll
        for (int j = 0; j < kNormRegs; ++j) {
            const int kq = tid + j * nt;
            if (kq < kq_end) sm.xn[m * nq + kq] = quad_norm<T>(sm.xn[m * nq + kq], r, nw.v[j]);
        }
        for (int kq = tid + kNormRegs * nt; kq < kq_end; kq += nt)
            sm.xn[m * nq + kq] = quad_norm<T>(sm.xn[m * nq + kq], r, load_norm4(a.norm_w, kq * 4));
    }
}

// Threads 0..127 own one (row r, column m) output of the 16 x 8 tile; `red`
// holds the 8 warps' partial tiles.  Partner rows (RoPE pairs, up / gate) are
// summed by the thread itself in the same warp order, so no second reduction
// pass (and no extra barrier) is needed.
__device__ __forceinline__ float tile_sum(const float *red, int r, int m) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) acc += red[(w * 16 + r) * 8 + m];
    return acc;
}

// Inputs of the epilogue other than the tile itself, for output row n and
// activation row m: the residual (RESID); the RoPE (cos, sin) pair at the
// row's position and the K/V cache offset of its token (QKV).
struct Side {
    float s0 = 0.f, s1 = 0.f;
    long off = 0;
};
__device__ __forceinline__ bool has_side(int epi) { return epi == EPI_RESID || epi == EPI_QKV || epi == EPI_ARESID; }
template <typename T>
__device__ __forceinline__ Side side_inputs(const GemvArgs &a, int n, int m) {
    Side s;
    if (a.epi == EPI_RESID || a.epi == EPI_ARESID) {
        s.s0 = to_float(reinterpret_cast<const T *>(a.res)[(long)m * a.ldr + n]);
    } else if (a.epi == EPI_QKV) {
        const int pos = a.pos[m];
        const bool rope = n < a.nq + a.nk;
        const int base = n < a.nq ? 0 : (rope ? a.nq : a.nq + a.nk);
        const int dd = (n - base) % a.hd;
        if (rope) {
            const float *f = a.freqs + (long)pos * a.hd + (dd & ~1);
            s.s0 = f[0];
            s.s1 = f[1];
        }
        if (n >= a.nq) {
            const long page = a.block_table[(long)a.seq[m] * a.max_pages + pos / a.page];
            s.off = ((page * a.kv_heads + (n - base) / a.hd) * a.page + pos % a.page) * a.hd + dd;
        }
    }
    return s;
}

// pre: the side inputs of this thread's (row, column), read before the wait
template <typename T>
__device__ void epilogue(const GemvArgs &a, const float *red, int tile, float &best_v, uint64_t &best_k,
                         const Side *pre) {
    const int tid = threadIdx.x;
    const int r = (tid >> 3) & 15, m = tid & 7;
    if (tid >= 128 || m >= a.M || !row_valid(a, tile, r)) return;
    const int n = tile_row(a, tile, r);
    const Side sd = pre ? *pre : has_side(a.epi) ? side_inputs<T>(a, n, m) : Side();
    float acc = tile_sum(red, r, m);
    switch (a.epi) {
    case EPI_STORE: {
        if (a.bias) acc += to_float(reinterpret_cast<const T *>(a.bias)[n]);
        reinterpret_cast<T *>(a.out)[(long)m * a.ldo + n] = from_float<T>(acc);
        break;
    }
    case EPI_RESID: {
        const float y = round_to<T>(acc);
        reinterpret_cast<T *>(a.out)[(long)m * a.ldo + n] = from_float<T>(sd.s0 + y);
        break;
    }
    case EPI_QKV: {
        const float y = round_to<T>(acc);
        if (n < a.nq + a.nk) {
            const float yp = round_to<T>(tile_sum(red, r ^ 1, m));
            const float cs = sd.s0, sn = sd.s1;
            const float o = (n & 1) ? (yp * sn + y * cs) : (y * cs - yp * sn);
            if (n < a.nq)
                reinterpret_cast<T *>(a.out)[(long)m * a.ldo + n] = from_float<T>(o);
            else
                reinterpret_cast<T *>(a.kpool)[sd.off] = from_float<T>(o);
        } else {
            reinterpret_cast<T *>(a.vpool)[sd.off] = from_float<T>(y);
        }
        break;
    }
    case EPI_SWIGLU: {
        if (r < 8) {
            const float u = round_to<T>(acc);
            const float gt = round_to<T>(tile_sum(red, r + 8, m));
            const float sig = 1.0f / (1.0f + expf(-gt));
            reinterpret_cast<T *>(a.out)[(long)m * a.ldo + tile * 8 + r] = from_float<T>((gt * sig) * u);
        }
        break;
    }
    case EPI_PARTIAL: {
        reinterpret_cast<float *>(a.out)[(long)m * a.ldo + n] = acc;
        break;
    }
    case EPI_LOGITS: {
        const float y = round_to<T>(acc);
        if (a.out) reinterpret_cast<T *>(a.out)[(long)m * a.ldo + n] = from_float<T>(y);
        // keys and the reference's row cut-off use the column in the whole vocabulary
        const long gn = (long)n + a.col_off;
        const long lim = (long)((a.n_total ? a.n_total : a.N) / a.pack) * a.pack;
        if (gn < lim && (y > best_v || (y == best_v && best_k != ~0ull))) {
            const uint64_t k = logits_key(gn, a.pack);
            if (y > best_v || k < best_k) {
                best_v = y;
                best_k = k;
            }
        }
        break;
    }
    }
}

// ARESID epilogue of one tile (all threads of the CTA take part): thread
// (row r, column m) pushes its fp32 partial sum, with the call's epoch for the
// tile, into every peer's buffer as one 8-byte word, then polls its own buffer
// until every peer's word for this (tile, r, m) carries the same epoch, adds
// the partials in rank order (so every rank computes the same x) and stores
// x = T(x + T(sum)), the RESID formula.  Payload slots alternate with the
// epoch's parity; a slot is rewritten two calls later, after every peer has
// pushed the call in between, which it does only once it has read this one.
// A wait that runs out records code 42 and leaves that output unchanged.
__device__ __forceinline__ void st_u64_sys(unsigned long long *p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_u64_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long ll_word(uint32_t bits, unsigned long long e) {
    return ((unsigned long long)(uint32_t)e << 32) | bits;
}
// Poll *p until its epoch half equals e; the value half, or false after limit_ns.
__device__ __forceinline__ bool ll_wait(const unsigned long long *p, unsigned long long e, uint32_t &bits,
                                        unsigned long long limit_ns) {
    unsigned long long v = ld_u64_sys(p);
    if ((uint32_t)(v >> 32) != (uint32_t)e) {
        const uint64_t t0 = globaltimer_ns();
        do {
            if (globaltimer_ns() - t0 > limit_ns) return false;
            v = ld_u64_sys(p);
        } while ((uint32_t)(v >> 32) != (uint32_t)e);
    }
    bits = (uint32_t)v;
    return true;
}

template <typename T>
__device__ void exchange_tile(const GemvArgs &a, const Smem &sm, int tile, const Side *pre, Timeline &tl) {
    const int tid = threadIdx.x;
    const TpLink &L = a.tp;
    unsigned long long *e_s = reinterpret_cast<unsigned long long *>(sm.misc + 8 + 128);
    if (tid == 0) {
        const unsigned long long e = L.tile_epoch[tile] + 1;
        L.tile_epoch[tile] = e;
        *e_s = e;
    }
    __syncthreads();
    const unsigned long long e = *e_s;
    // word (parity, tile, source rank, tid) of a receiver's buffer; only the
    // words of real outputs (activation rows m < M, rows inside N) are pushed
    // and awaited -- at batch 1, 16 of the tile's 128
    const size_t base = ((size_t)(e & 1) * kTpMaxTiles + tile) * kTpMaxWorld * 128 + tid;
    const int r = (tid >> 3) & 15, m = tid & 7;
    const bool valid = tid < 128 && m < a.M && row_valid(a, tile, r);
    float own = 0.f;
    if (valid) {
        own = tile_sum(sm.red, r, m);
        const unsigned long long w = ll_word(__float_as_uint(own), e);
        for (int q = 0; q < L.world; ++q)
            if (q != L.rank)
                st_u64_sys(reinterpret_cast<unsigned long long *>(L.peers[q] + kXTileLL) + base + L.rank * 128, w);
    }
    tl.phase(5);  // first tile pushed
    __syncthreads();  // e_s is rewritten by the next tile
    if (!valid) return;
    const unsigned long long *mine = reinterpret_cast<const unsigned long long *>(L.peers[L.rank] + kXTileLL) + base;
    float acc = 0.f;
    bool ok = true;
    for (int q = 0; q < L.world; ++q) {
        if (q == L.rank) {
            acc += own;
            continue;
        }
        uint32_t bits = 0;
        if (!ll_wait(mine + q * 128, e, bits, L.limit_ns)) {
            ok = false;
            break;
        }
        acc += __uint_as_float(bits);
    }
    if (!ok) {
        atomicCAS(a.err, 0, 42);
        return;
    }
    const int n = tile_row(a, tile, r);
    const float res = pre ? pre->s0 : to_float(reinterpret_cast<const T *>(a.res)[(long)m * a.ldr + n]);
    reinterpret_cast<T *>(a.out)[(long)m * a.ldo + n] = from_float<T>(res + round_to<T>(acc));
}

// The logits winners of a vocabulary shard (tid < M hold this rank's best
// value and order key of row tid) exchanged with every rank by the last CTA,
// in the same push protocol (three words per row: value, key low, key high);
// the best over ranks in the reference argmax's tie order gives the token.
// All threads of the CTA call it.
__device__ void exchange_winners(const GemvArgs &a, float bv, uint64_t bk) {
    const int tid = threadIdx.x;
    const TpLink &L = a.tp;
    __shared__ unsigned long long e_w;
    if (tid == 0) {
        e_w = *L.win_epoch + 1;
        *L.win_epoch = e_w;
    }
    __syncthreads();
    if (tid >= a.M) return;
    const unsigned long long e = e_w;
    // word (parity, source rank, row, j) of a receiver's buffer
    auto slot = [&](int src) { return ((size_t)(e & 1) * kTpMaxWorld + src) * 32 + tid * 4; };
    const unsigned long long w0 = ll_word(__float_as_uint(bv), e), w1 = ll_word((uint32_t)bk, e),
                             w2 = ll_word((uint32_t)(bk >> 32), e);
    for (int q = 0; q < L.world; ++q) {
        if (q == L.rank) continue;
        unsigned long long *d = reinterpret_cast<unsigned long long *>(L.peers[q] + kXWinLL) + slot(L.rank);
        st_u64_sys(d, w0);
        st_u64_sys(d + 1, w1);
        st_u64_sys(d + 2, w2);
    }
    float best_v = -INFINITY;
    uint64_t best_k = ~0ull;
    const unsigned long long *mine = reinterpret_cast<const unsigned long long *>(L.peers[L.rank] + kXWinLL);
    for (int q = 0; q < L.world; ++q) {
        float v = bv;
        uint64_t k = bk;
        if (q != L.rank) {
            uint32_t b0 = 0, b1 = 0, b2 = 0;
            if (!ll_wait(mine + slot(q), e, b0, L.limit_ns) || !ll_wait(mine + slot(q) + 1, e, b1, L.limit_ns) ||
                !ll_wait(mine + slot(q) + 2, e, b2, L.limit_ns)) {
                atomicCAS(a.err, 0, 43);
                return;
            }
            v = __uint_as_float(b0);
            k = ((uint64_t)b2 << 32) | b1;
        }
        if (k == ~0ull) continue;
        if (v > best_v || (v == best_v && k < best_k)) {
            best_v = v;
            best_k = k;
        }
    }
    a.tokens[tid] = logits_index(best_k, a.pack);
}

// Epilogue of a tile owned by one warp (SwiGLU or logits): lane (g, t) has
// rows g, g + 8 for columns 2t, 2t + 1 (SwiGLU: up row g, gate row g + 8).
template <typename T>
__device__ __forceinline__ void warp_epilogue(const GemvArgs &a, int tile, int g, int t, const float (&c)[2][4],
                                              float (&bv)[2], uint64_t (&bk)[2]) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int m = 2 * t + j;
        const float lo = c[0][j] + c[1][j], hi = c[0][2 + j] + c[1][2 + j];
        if (m >= a.M) continue;
        if (a.epi == EPI_SWIGLU) {
            if (tile * 8 + g < a.F) {
                const float u = round_to<T>(lo);
                const float gt = round_to<T>(hi);
                const float sig = 1.0f / (1.0f + expf(-gt));
                reinterpret_cast<T *>(a.out)[(long)m * a.ldo + tile * 8 + g] = from_float<T>((gt * sig) * u);
            }
        } else {  // EPI_LOGITS
            const long lim = (long)((a.n_total ? a.n_total : a.N) / a.pack) * a.pack;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int n = tile * kTileRows + g + 8 * h;
                if (n >= a.N) continue;
                const float y = round_to<T>(h ? hi : lo);
                if (a.out) reinterpret_cast<T *>(a.out)[(long)m * a.ldo + n] = from_float<T>(y);
                const long gn = (long)n + a.col_off;
                if (gn < lim && (y > bv[j] || (y == bv[j] && bk[j] != ~0ull))) {
                    const uint64_t k = logits_key(gn, a.pack);
                    if (y > bv[j] || k < bk[j]) {
                        bv[j] = y;
                        bk[j] = k;
                    }
                }
            }
        }
    }
}

template <typename T, int WT, int NS>
__global__ void __launch_bounds__(kWarps * 32, 2) gemv_kernel(const __grid_constant__ GemvArgs a) {
    Timeline tl;
    using F = WFmt<WT>;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const int nchunks = (a.K + F::kChunk - 1) / F::kChunk;
    const int Kpad = nchunks * F::kChunk;
    Smem sm;
    sm.ring = smem_raw;
    sm.bars = reinterpret_cast<uint64_t *>(sm.ring + (size_t)kWarps * NS * kStageBytes);
    sm.xn = reinterpret_cast<uint2 *>(sm.bars + kWarps * NS);
    // X goes to shared memory when normalised here, or when small enough
    const bool stage = a.norm_w || (size_t)a.M * Kpad * 2 <= kXStageMax;
    sm.red = reinterpret_cast<float *>(sm.xn + (stage ? (size_t)(Kpad / 4) * a.M : 0));
    sm.misc = sm.red + kWarps * 16 * 8;
    if (stage) {
        sm.xsrc = sm.xn;
        sm.xld = Kpad / 4;
    } else {
        sm.xsrc = reinterpret_cast<const uint2 *>(a.x);
        sm.xld = a.ldx / 4;
    }

    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = num_tiles(a);
    const bool tma = a.bulk != 0;
    if (threadIdx.x < kWarps * NS) mbar_init(sm.bars + threadIdx.x, 1);
    mbar_fence_init();
    __syncthreads();
    if (threadIdx.x == 32 && a.pf) l2_prefetch_slice(a.pf, a.pf_bytes, blockIdx.x, gridDim.x);

    // this warp's unit sequence.  CTA tiles: tiles blockIdx.x, +gridDim.x, ...,
    // chunks w, w + 8, ...; warp tiles: tiles gw, gw + 8 gridDim.x, ..., all chunks
    const bool wmode = warp_tiles(a.epi, ntiles, a.warp_tile_min);
    const int gw = blockIdx.x * kWarps + w, nw = gridDim.x * kWarps;
    const int cstart = wmode ? 0 : w, cstep = wmode ? 1 : kWarps, tstep = wmode ? nw : (int)gridDim.x;
    int p_tile = wmode ? gw : (int)blockIdx.x, p_chunk = cstart;  // producer cursor
    const bool has_work = wmode || w < nchunks;  // a warp with no chunk in this K idles in the k-loop
    if (tma)
        for (int s = 0; s < NS; ++s)
            produce_unit<WT>(a, sm, w, s, lane, has_work, ntiles, nchunks, p_tile, p_chunk, cstart, cstep, tstep, NS);
    // Inputs that the previous kernel does not write are read before the wait:
    // the RMSNorm weights, and with a.pre the side inputs of this CTA's first
    // tile (written two or more launches back).
    NormW normw;
    if (stage && a.norm_w) norm_pre(a, normw);
    Side side0;
    const bool pre = a.pre && !wmode && has_side(a.epi) && (int)blockIdx.x < ntiles;
    if (pre) {
        const int r = (threadIdx.x >> 3) & 15, m = threadIdx.x & 7;
        if (threadIdx.x < 128 && m < a.M && row_valid(a, blockIdx.x, r))
            side0 = side_inputs<T>(a, tile_row(a, blockIdx.x, r), m);
    }
    // weights are in flight; wait for the producer of X, then let the next kernel
    // in the stream start its own weight prefetch
    pdl_wait();
    pdl_trigger();
    tl.mark(a.epi, a.N, a.K);
    if (stage) stage_xn<T>(a, sm, Kpad, normw);
    __syncthreads();
    tl.phase(0);  // activations staged (and normalised)

    float best_v = -INFINITY;
    uint64_t best_k = ~0ull;
    int consumed = 0;
    bool ok = true;
    if (wmode) {
        // lane (g, t) holds rows g, g + 8 and columns 2t, 2t + 1 of each of its tiles
        const int g = lane >> 2, t = lane & 3;
        float bv[2] = {-INFINITY, -INFINITY};
        uint64_t bk[2] = {~0ull, ~0ull};
        for (int tile = gw; tile < ntiles; tile += nw) {
            float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
            for (int chunk = 0; chunk < nchunks; ++chunk) {
                const int slot = consumed % NS;
                if (tma) {
                    if (!mbar_wait_bounded(sm.bars + w * NS + slot, (consumed / NS) & 1, a.err, 1))
                        ok = false;
                } else {
                    issue_unit<WT>(a, sm, w, slot, tile, chunk, lane, false, NS);
                    __syncwarp();
                }
                if (ok) consume_unit<WT>(a, sm, w, slot, chunk, lane, c, NS);
                __syncwarp();
                ++consumed;
                if (tma && ok)
                    produce_unit<WT>(a, sm, w, slot, lane, has_work, ntiles, nchunks, p_tile, p_chunk, cstart, cstep,
                                     tstep, NS);
            }
            warp_epilogue<T>(a, tile, g, t, c, bv, bk);
        }
        if (a.epi == EPI_LOGITS) {
            // best of the 8 lanes that share t, then one (value, key) per warp and column
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv[j], o);
                    const uint64_t okey = __shfl_xor_sync(0xffffffffu, bk[j], o);
                    if (ov > bv[j] || (ov == bv[j] && okey < bk[j])) {
                        bv[j] = ov;
                        bk[j] = okey;
                    }
                }
            float *sv = sm.misc + 8;
            uint64_t *sk = reinterpret_cast<uint64_t *>(sm.misc + 8 + 128);
            if (g == 0) {
                sv[w * 8 + 2 * t] = bv[0];
                sk[w * 8 + 2 * t] = bk[0];
                sv[w * 8 + 2 * t + 1] = bv[1];
                sk[w * 8 + 2 * t + 1] = bk[1];
            }
        }
        __syncthreads();
    }
    for (int tile = blockIdx.x; !wmode && tile < ntiles; tile += gridDim.x) {
        float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        if (has_work) {
            for (int chunk = w; chunk < nchunks; chunk += kWarps) {
                const int slot = consumed % NS;
                if (tma) {
                    // a box that never lands is reported (bounded wait), not waited on forever
                    if (!mbar_wait_bounded(sm.bars + w * NS + slot, (consumed / NS) & 1, a.err, 1))
                        ok = false;
                } else {
                    issue_unit<WT>(a, sm, w, slot, tile, chunk, lane, false, NS);
                    __syncwarp();
                }
                if (w == 0) tl.phase(1);  // first unit landed
                if (ok) consume_unit<WT>(a, sm, w, slot, chunk, lane, c, NS);
                __syncwarp();  // the slot is free again
                if (w == 0) tl.phase(2);  // first unit consumed
                ++consumed;
                if (tma && ok)
                    produce_unit<WT>(a, sm, w, slot, lane, has_work, ntiles, nchunks, p_tile, p_chunk, cstart, cstep,
                                     tstep, NS);
            }
        }
        // partial tile of this warp -> shared memory (rows g, g+8; columns 2t, 2t+1)
        const int g = lane >> 2, t = lane & 3;
        float *red = sm.red + w * 16 * 8;
        red[g * 8 + 2 * t] = c[0][0] + c[1][0];
        red[g * 8 + 2 * t + 1] = c[0][1] + c[1][1];
        red[(g + 8) * 8 + 2 * t] = c[0][2] + c[1][2];
        red[(g + 8) * 8 + 2 * t + 1] = c[0][3] + c[1][3];
        __syncthreads();
        if (a.epi == EPI_ARESID)
            exchange_tile<T>(a, sm, tile, pre && tile == (int)blockIdx.x ? &side0 : nullptr, tl);
        else
            epilogue<T>(a, sm.red, tile, best_v, best_k, pre && tile == (int)blockIdx.x ? &side0 : nullptr);
        __syncthreads();  // red is rewritten by the next tile
        tl.phase(3);          // first tile stored
    }

    tl.phase(4);  // all tiles
    if (a.epi == EPI_LOGITS) {
        // per-CTA argmax partials: reduce over the 16 row-threads of each column m
        const int tid = threadIdx.x, m = tid & 7;
        float *sv = sm.misc + 8;                                        // [16][8] or [8 warps][8]
        uint64_t *sk = reinterpret_cast<uint64_t *>(sm.misc + 8 + 128);  // (written above in warp mode)
        if (!wmode && tid < 128) {
            sv[tid] = best_v;
            sk[tid] = best_k;
        }
        __syncthreads();
        if (tid < 8 && tid < a.M) {
            float v = sv[tid];
            uint64_t k = sk[tid];
            for (int r = 1; r < (wmode ? kWarps : 16); ++r) {
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
        (void)m;
        // the last CTA to finish reduces the partials to token ids
        __shared__ int last;
        __threadfence();
        __syncthreads();
        if (tid == 0) last = (atomicAdd(a.counter, 1) == (int)gridDim.x - 1);
        __syncthreads();
        if (last) {
            // The best (value, key) is a maximum over a total order, so any
            // reduction tree gives the same winner: 32 groups of 8 threads (one
            // per activation row) take every 32nd CTA's partial, then the 4
            // groups of a warp and the 8 warps are combined.
            __threadfence();
            const int mrow = tid & 7, grp = tid >> 3, wid = tid >> 5, lane = tid & 31;
            float bv = -INFINITY;
            uint64_t bk = ~0ull;
            auto take = [&](float ov, uint64_t okey) {
                if (ov > bv || (ov == bv && okey < bk)) {
                    bv = ov;
                    bk = okey;
                }
            };
            for (int b0 = grp; b0 < (int)gridDim.x; b0 += 32 * 4) {
                float ov[4];
                uint64_t okey[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int b = b0 + u * 32;
                    ov[u] = b < (int)gridDim.x ? __ldcg(a.part_val + (long)b * 8 + mrow) : -INFINITY;
                    okey[u] = b < (int)gridDim.x ? __ldcg(a.part_key + (long)b * 8 + mrow) : ~0ull;
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) take(ov[u], okey[u]);
            }
#pragma unroll
            for (int o = 8; o < 32; o <<= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const uint64_t okey = __shfl_xor_sync(0xffffffffu, bk, o);
                take(ov, okey);
            }
            if (lane < 8) {
                sv[wid * 8 + lane] = bv;
                sk[wid * 8 + lane] = bk;
            }
            __syncthreads();
            if (tid < a.M) {
                bv = -INFINITY;
                bk = ~0ull;
                for (int w = 0; w < kWarps; ++w) take(sv[w * 8 + tid], sk[w * 8 + tid]);
                if (a.tokens && a.tp.world == 1) a.tokens[tid] = logits_index(bk, a.pack);
                if (a.best_val) {
                    a.best_val[tid] = bv;
                    a.best_key[tid] = bk;
                }
            }
            if (tid == 0) *a.counter = 0;
            if (a.tp.world > 1 && a.tokens) exchange_winners(a, bv, bk);
        }
    }
}

size_t gemv_smem_bytes(int K, int M, int wt, bool norm, int ns = kStages) {
    const int chunk = (wt == kQ8_0 || wt == kQ4_0) ? 256 : WFmt<kF16>::kChunk;
    const int Kpad = (K + chunk - 1) / chunk * chunk;
    const bool stage = norm || (size_t)M * Kpad * 2 <= kXStageMax;
    return (size_t)kWarps * ns * kStageBytes + kWarps * ns * 8 + (stage ? (size_t)Kpad * M * 2 : 0) +
           kWarps * 16 * 8 * 4 +
           (8 + 128) * 4 + 128 * 8;
}

template <typename T, int WT, int NS> void launch(const GemvArgs &a, int grid, size_t smem, cudaStream_t s, bool pdl) {
    auto kern = gemv_kernel<T, WT, NS>;
    // raise the dynamic shared-memory limit only when a launch needs more
    static int configured = 0;
    if ((int)smem > configured) {
        WK_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        configured = (int)smem;
    }
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
    if (wtype == kQ8_0 || wtype == kQ4_0) return act == kF16 && K % 32 == 0;
    if (wtype == kF16) return act == kF16 && K % 16 == 0;
    if (wtype == kBF16) return act == kBF16 && K % 16 == 0;
    return false;
}

void gemv(GemvArgs a, int act, cudaStream_t s) {
    if (a.M <= 0 || a.M > 8) WK_PANIC("gemv: M=%d outside [1, 8]", a.M);
    if (a.epi == EPI_ARESID && (a.tp.world < 2 || !a.tp.peers || (a.N + kTileRows - 1) / kTileRows > kTpMaxTiles))
        WK_PANIC("gemv: the all-reduce epilogue needs the peer exchange and at most %d tiles", kTpMaxTiles);
    if (!gemv_supported(a.wtype, act, a.K)) WK_PANIC("gemv: unsupported wtype %d / act %d / K %d", a.wtype, act, a.K);
    const long rb = quant_row_bytes(a.wtype, a.K);
    // weight tiles stream by TMA when rows are 16-byte aligned
    const CUtensorMap *map = nullptr;
    if (((uintptr_t)a.w % 16 == 0) && (rb % 16 == 0)) {
        const int box_inner = a.wtype == kQ8_0   ? WFmt<kQ8_0>::kRowB / 2
                              : a.wtype == kQ4_0 ? WFmt<kQ4_0>::kRowB / 2
                                                 : WFmt<kF16>::kRowB / 2;
        const long rows = a.epi == EPI_SWIGLU ? 2L * a.F : (long)a.N;
        map = weight_map(a.w, rows, rb, box_inner, a.epi == EPI_SWIGLU ? 8 : kTileRows);
    }
    a.bulk = map ? 1 : 0;
    a.warp_tile_min = g_rt.warp_tile_min;
    if (map) a.wmap = *map;
    if (!a.err) a.err = g_rt.d_error;
    if (((uintptr_t)a.x % 8) || (a.ldx % 4)) WK_PANIC("gemv: activations must be 8-byte aligned rows");
    const size_t smem = gemv_smem_bytes(a.K, a.M, a.wtype, a.norm_w != nullptr);
    if ((int)smem > g_rt.max_smem_optin) {
        // the normalised X does not fit beside the ring: split the activation rows
        if (a.M == 1) WK_PANIC("gemv: K=%d needs %zu B of shared memory", a.K, smem);
        const int m1 = a.M / 2;
        const size_t es = act == kF32 ? 4 : 2;
        GemvArgs b = a;
        b.M = a.M - m1;
        a.M = m1;
        b.x = (const char *)a.x + (size_t)m1 * a.ldx * es;
        if (b.epi != EPI_LOGITS) b.out = (char *)a.out + (size_t)m1 * a.ldo * (b.epi == EPI_PARTIAL ? 4 : es);
        if (b.res) b.res = (const char *)a.res + (size_t)m1 * a.ldr * es;
        if (b.pos) b.pos += m1;
        if (b.seq) b.seq += m1;
        if (b.tokens) b.tokens += m1;
        if (b.best_val) {
            b.best_val += m1;
            b.best_key += m1;
        }
        if (b.epi == EPI_LOGITS && b.out) b.out = (char *)a.out + (size_t)m1 * a.ldo * es;
        gemv(a, act, s);
        gemv(b, act, s);
        return;
    }
    const int ntiles = a.epi == EPI_SWIGLU ? (a.F + 7) / 8 : (a.N + kTileRows - 1) / kTileRows;
    // two CTAs per SM when both fit (about 200 KB of weight tiles in flight per
    // SM); when the 3-stage rings do not fit twice, 2-stage rings that do are
    // preferred (16 warps per SM hide more latency than deeper rings)
    size_t smem_used = smem;
    int ns = kStages;
    // 2-stage rings only where they buy a second CTA per SM: a launch of at most one tile per SM
    // whose warps stream more units than 2 slots hold (e.g. a 2048-row down projection over
    // K = 8192: 128 tiles, 4 units per warp) keeps 3 (1B decode 0.690 -> 0.649 ms/step; 6 slots,
    // 231 KB, measured 0.711)
    const int units = (a.K / 256 + kWarps - 1) / kWarps;  // per warp and tile (CTA tiles)
    const bool one_per_sm = ntiles <= g_rt.num_sms && units > 2;
    if (!one_per_sm && 2 * (smem + 1024) > (size_t)g_rt.smem_per_sm) {
        const size_t smem2 = gemv_smem_bytes(a.K, a.M, a.wtype, a.norm_w != nullptr, 2);
        if (2 * (smem2 + 1024) <= (size_t)g_rt.smem_per_sm) {
            smem_used = smem2;
            ns = 2;
        }
    }
    const int per_sm = 2 * (smem_used + 1024) <= (size_t)g_rt.smem_per_sm ? 2 : 1;
    int grid = ntiles < g_rt.num_sms * per_sm ? ntiles : g_rt.num_sms * per_sm;
    if (a.epi == EPI_LOGITS && grid > kMaxLogitCtas) grid = kMaxLogitCtas;
    const bool pdl = g_rt.pdl && a.pdl;
    if (ns == 2) {
        if (a.wtype == kQ8_0)
            launch<__half, kQ8_0, 2>(a, grid, smem_used, s, pdl);
        else if (a.wtype == kQ4_0)
            launch<__half, kQ4_0, 2>(a, grid, smem_used, s, pdl);
        else if (a.wtype == kF16)
            launch<__half, kF16, 2>(a, grid, smem_used, s, pdl);
        else
            launch<__nv_bfloat16, kBF16, 2>(a, grid, smem_used, s, pdl);
    } else {
        if (a.wtype == kQ8_0)
            launch<__half, kQ8_0, kStages>(a, grid, smem_used, s, pdl);
        else if (a.wtype == kQ4_0)
            launch<__half, kQ4_0, kStages>(a, grid, smem_used, s, pdl);
        else if (a.wtype == kF16)
            launch<__half, kF16, kStages>(a, grid, smem_used, s, pdl);
        else
            launch<__nv_bfloat16, kBF16, kStages>(a, grid, smem_used, s, pdl);
    }
}

#ifdef WK_TIMELINE
void timeline_bind_gemv(const TimelineBuf &b) { WK_CHECK(cudaMemcpyToSymbol(c_tl, &b, sizeof b)); }
#else
void timeline_bind_gemv(const TimelineBuf &) {}
#endif

}  // namespace wk
