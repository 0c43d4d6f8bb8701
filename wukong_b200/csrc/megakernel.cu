// The engine's decode step (batch <= 8, Q8_0 weights, fp16 activations) as one
// persistent cooperative kernel: one CTA per SM runs every phase of the step
//
//   embed -> per layer { qkv GEMV [RMSNorm | RoPE + KV append] | attention |
//   o GEMV [+x] | fc GEMV [RMSNorm | SwiGLU] | down GEMV [+x] } -> logits GEMV
//   [RMSNorm | argmax] -> token, advance
//
// with a grid-wide barrier between phases (82 for 16 layers) instead of 83
// kernel launches.  The point is the weight stream: each warp owns a ring of
// 16-row x 256-value Q8_0 tiles (one 2-D TMA box each) and walks a fixed
// schedule of (phase, tile, chunk) units for the whole step, requesting the
// next unit as soon as a slot frees.  Weights do not depend on activations, so
// while a CTA waits at a barrier (or runs attention) its rings keep filling
// with the next phases' tiles and DRAM never idles between kernels.
//
// The arithmetic is the multi-kernel path's, unit for unit: the same tile and
// chunk split over the 8 warps, the same mma.sync dequantised products, the
// same RMSNorm staging, epilogues and attention rounding points (reference
// semantics of cuda.cu:1095-1111, :533-601, :207-236, :767-852, :176-205,
// :423-435, :480-531), so tokens and activations equal the graph path's.
//
// Inter-CTA data (activations, the newest K/V row, positions, partials) is
// read through L2 (ld.global.cg / cp.async.cg).  Every barrier wait is
// bounded: a CTA that waits more than one second records an error code, marks
// the barrier aborted (all later waits pass at once) and the kernel runs to
// its end; the host reports the error word after its next synchronisation.
#include "common.cuh"
#include "wukong_internal.cuh"

namespace wk {

namespace {

constexpr int kW = 8;                // warps per CTA (all compute; each streams its own weight units)
constexpr int kThreads = kW * 32;
constexpr int kRowB = 272;           // bytes of 256 Q8_0 values (8 blocks)
constexpr int kUnit = 16 * kRowB;    // one (tile, chunk) unit: 16 rows
constexpr int kPg = 64;              // KV page (tokens)
constexpr int kPgSlots = 4;          // KV pages in flight in the attention phase
constexpr unsigned long long kAbort = 1ull << 63;  // set in the barrier counter by a wait that gave up
enum : int { MK_QKV = 0, MK_O = 1, MK_FC = 2, MK_DOWN = 3, MK_LOGITS = 4 };

struct Gp {
    int kind, ntiles, nchunks;
    bool wm;  // one tile per warp (warp_tiles), else split over the CTA's warps by K-chunk
};

// GEMV phase gi of the step: 4 l + kind for layer l, 4 L for the logits
__device__ __forceinline__ Gp gp_of(const MkArgs &a, int gi) {
    Gp p;
    int K;
    if (gi >= 4 * a.L) {
        p.kind = MK_LOGITS;
        p.ntiles = (a.V + 15) / 16;
        K = a.d;
    } else {
        p.kind = gi & 3;
        switch (p.kind) {
        case MK_QKV:
            p.ntiles = ((a.H + 2 * a.Hk) * a.D + 15) / 16;
            K = a.d;
            break;
        case MK_O:
            p.ntiles = (a.d + 15) / 16;
            K = a.H * a.D;
            break;
        case MK_FC:
            p.ntiles = a.F / 8;  // 8 up rows + the 8 matching gate rows
            K = a.d;
            break;
        default:
            p.ntiles = (a.d + 15) / 16;
            K = a.F;
        }
    }
    p.nchunks = K / 256;
    p.wm = warp_tiles(p.kind == MK_FC ? EPI_SWIGLU : (p.kind == MK_LOGITS ? EPI_LOGITS : EPI_STORE), p.ntiles,
                      a.warp_tile_min);
    return p;
}

// Producer cursor over this warp's units of the whole step, in consumption
// order: phases in order; in CTA-split phases this CTA's tiles (round-robin
// over the CTAs, continuing from the previous such phase) and chunks w, w + 8,
// ...; in warp-tile phases this warp's tiles (round-robin over all warps) and
// every chunk.
struct Cursor {
    int gi, tile, chunk, ntiles, nchunks, kind, off, offw;
    bool wm;
};

__device__ __forceinline__ int first_tile(int off) {
    const int G = gridDim.x;
    return ((int)blockIdx.x - off % G + G) % G;
}
__device__ __forceinline__ int first_tile_w(int offw, int w) {
    const int NW = gridDim.x * kW;
    return ((int)blockIdx.x * kW + w - offw % NW + NW) % NW;
}

__device__ __forceinline__ void cur_seek(const MkArgs &a, Cursor &c, int w) {
    const int last = 4 * a.L;
    while (c.gi <= last) {
        const Gp p = gp_of(a, c.gi);
        c.ntiles = p.ntiles;
        c.nchunks = p.nchunks;
        c.kind = p.kind;
        c.wm = p.wm;
        const int t0 = p.wm ? first_tile_w(c.offw, w) : first_tile(c.off);
        if ((p.wm || w < p.nchunks) && t0 < p.ntiles) {
            c.tile = t0;
            c.chunk = p.wm ? 0 : w;
            return;
        }
        if (p.wm)
            c.offw = (c.offw + p.ntiles) % (int)(gridDim.x * kW);
        else
            c.off = (c.off + p.ntiles) % (int)gridDim.x;
        ++c.gi;
    }
}

__device__ __forceinline__ void cur_next(const MkArgs &a, Cursor &c, int w) {
    c.chunk += c.wm ? 1 : kW;
    if (c.chunk < c.nchunks) return;
    c.tile += c.wm ? (int)gridDim.x * kW : (int)gridDim.x;
    if (c.tile < c.ntiles) {
        c.chunk = c.wm ? 0 : w;
        return;
    }
    if (c.wm)
        c.offw = (c.offw + c.ntiles) % (int)(gridDim.x * kW);
    else
        c.off = (c.off + c.ntiles) % (int)gridDim.x;
    ++c.gi;
    cur_seek(a, c, w);
}

__device__ __forceinline__ void tma_box(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"((uint64_t)map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Weight tensor maps of the model being decoded, in the constant bank (the TMA
// unit reads a descriptor per copy; constant memory serves it from the
// constant cache).  Filled by mk_launch when the model changes.
constexpr int kMaxMaps = 4 * 112 + 1;  // 112 layers
__constant__ CUtensorMap c_maps[kMaxMaps];

struct Sm {
    uint8_t *ring;   // [kW][S][kUnit]
    uint64_t *bars;  // [kW][S]
    float *red;      // [2][kW][16][8] partial tiles, alternating per tile
    float *misc;     // [8] norm scales, [128] logits values, then [128] u64 keys
    uint8_t *work;   // normalised X [B][d] half, or the attention buffers
};

__device__ __forceinline__ void issue_unit(const MkArgs &a, const Sm &sm, const Cursor &c, int w, int S, int slot) {
    uint8_t *dst = sm.ring + (size_t)(w * S + slot) * kUnit;
    uint64_t *bar = sm.bars + w * S + slot;
    const CUtensorMap *map = c_maps + c.gi;
    mbar_expect_tx(bar, kUnit);
    const int x = c.chunk * (kRowB / 2);  // uint16 column of the box
    if (c.kind == MK_FC) {
        tma_box(dst, map, x, c.tile * 8, bar);
        tma_box(dst + 8 * kRowB, map, x, a.F + c.tile * 8, bar);
    } else {
        tma_box(dst, map, x, c.tile * 16, bar);
    }
}

__device__ __forceinline__ float ldcg_h(const __half *p) {
    return __half2float(__ushort_as_half(__ldcg(reinterpret_cast<const unsigned short *>(p))));
}

// ---------------------------------------------------------------- grid barrier
__device__ __forceinline__ unsigned long long ld_acquire(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Grid-wide barrier on a monotonic 64-bit counter: launch k of the engine
// starts at a.bar_base (the arrivals of all earlier launches), so the counter
// is never reset.
__device__ __forceinline__ void grid_sync(const MkArgs &a, unsigned long long target, int code) {
    __syncthreads();
    if (threadIdx.x == 0) {
        // arrive without waiting for the reply (release orders this CTA's writes before it)
        asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(a.bar), "l"(1ull) : "memory");
        unsigned long long v = ld_acquire(a.bar);
        if (v < target && !(v & kAbort)) {
            const uint64_t t0 = globaltimer_ns();
            while (true) {
                __nanosleep(100);
                v = ld_acquire(a.bar);
                if (v >= target || (v & kAbort)) break;
                if (globaltimer_ns() - t0 > 1000000000ull) {
                    atomicCAS(a.err, 0, code);
                    atomicOr(a.bar, kAbort);
                    break;
                }
            }
        }
        __threadfence();
    }
    __syncthreads();
}

// ---------------------------------------------------------------- phases
// x[b] = token_embd[ids[b]] converted to half (cuda.cu:238-252)
__device__ void mk_embed(const MkArgs &a) {
    const long total = (long)a.B * a.d;
    for (long i = (long)blockIdx.x * kThreads + threadIdx.x; i < total; i += (long)gridDim.x * kThreads) {
        const int b = (int)(i / a.d), k = (int)(i - (long)b * a.d);
        long id = a.ids[b];
        if (id < 0 || id >= a.vocab_total) {
            if (k == 0) atomicCAS(a.err, 0, 2);
            id = 0;
        }
        float v;
        if (a.embd_type == kQ8_0) {
            const uint8_t *blk = a.embd + (id * (a.d / 32) + k / 32) * 34;
            const float s = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
            v = __half2float(__float2half_rn(s * (float)(int8_t)blk[2 + (k & 31)]));
        } else if (a.embd_type == kF16) {
            v = __half2float(reinterpret_cast<const __half *>(a.embd)[id * a.d + k]);
        } else if (a.embd_type == kBF16) {
            v = __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(a.embd)[id * a.d + k]);
        } else {
            v = reinterpret_cast<const float *>(a.embd)[id * a.d + k];
        }
        a.x[i] = __float2half_rn(v);
    }
}

// RMSNorm of x rows into shared memory, rounded to half (cuda.cu:533-601).
// x is copied in with 16-byte loads first (one L2 round trip), then the sums
// of squares run over shared memory in the GEMV prologue's order, so the
// result is bit-identical to it.
__device__ void mk_stage_norm(const MkArgs &a, const Sm &sm, const float *nw) {
    const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint4 *raw = reinterpret_cast<uint4 *>(sm.work);
    const uint4 *xg = reinterpret_cast<const uint4 *>(a.x);
    const int n16 = a.B * a.d / 8;
    for (int i = threadIdx.x; i < n16; i += kThreads) raw[i] = __ldcg(xg + i);
    __syncthreads();
    // sums of squares in the GEMV prologue's order: thread t adds the quads
    // t, t + 256, ... of a row, its warp sums by butterfly, then the 8 warps'
    // sums are added in warp order
    __shared__ float wsum[kW * 8];
    const int nq = a.d / 4;
    uint2 *xs = reinterpret_cast<uint2 *>(sm.work);
    for (int m = 0; m < a.B; ++m) {
        float ss = 0.f;
        for (int kq = threadIdx.x; kq < nq; kq += kThreads) {
            const uint2 r = xs[m * nq + kq];
            const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(&r.x));
            const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(&r.y));
            ss += lo.x * lo.x;
            ss += lo.y * lo.y;
            ss += hi.x * hi.x;
            ss += hi.y * hi.y;
        }
        ss = warp_sum(ss);
        if (lane == 0) wsum[wid * 8 + m] = ss;
    }
    __syncthreads();
    if (threadIdx.x < a.B) {
        float tot = 0.f;
        for (int w = 0; w < kW; ++w) tot += wsum[w * 8 + threadIdx.x];
        sm.misc[threadIdx.x] = rsqrtf(tot / (float)a.d + a.eps);
    }
    __syncthreads();
    // normalise in place: every thread rewrites the 4 values it read
    for (int i = threadIdx.x; i < nq * a.B; i += kThreads) {
        const int m = i / nq, k = (i - m * nq) * 4;
        const uint2 r = xs[i];
        const float4 wv = *reinterpret_cast<const float4 *>(nw + k);
        const float sc = sm.misc[m];
        const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(&r.x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(&r.y));
        const __half2 o0 = __floats2half2_rn((lo.x * sc) * wv.x, (lo.y * sc) * wv.y);
        const __half2 o1 = __floats2half2_rn((hi.x * sc) * wv.z, (hi.y * sc) * wv.w);
        xs[i] = make_uint2(h2_as_u32(o0), h2_as_u32(o1));
    }
    __syncthreads();
}

// One unit (16 rows x 256 k) into the 16 x 8 accumulator; X fragments from
// shared memory or (o / down inputs) from global memory through L2.
template <bool kGlobal>
__device__ __forceinline__ void mk_consume(const uint8_t *st, const uint2 *xbase, long xld, int chunk, int B, int lane,
                                           float (&c)[2][4]) {
    const int g = lane >> 2, t = lane & 3;
    const uint8_t *r0 = st + g * kRowB;
    const uint8_t *r1 = st + (g + 8) * kRowB;
    const bool has_x = g < B;
    const uint2 *xl = xbase + (long)(has_x ? g : 0) * xld + (long)chunk * 64 + t;  // 256 k = 64 uint2
    uint2 xv[16];
#pragma unroll
    for (int s = 0; s < 16; ++s) {
        uint2 v = kGlobal ? __ldcg(xl + 4 * s) : xl[4 * s];
        xv[s] = has_x ? v : make_uint2(0u, 0u);
    }
#pragma unroll
    for (int b = 0; b < 8; ++b) q8_block(r0, r1, b * 34, (b & 1) != 0, t, xv[2 * b], xv[2 * b + 1], c);
}

// Epilogue of a tile owned by one warp (SwiGLU or logits); lane (g, t) has
// rows g, g + 8 for columns 2t, 2t + 1.  Same arithmetic as the per-op GEMV.
__device__ __forceinline__ void mk_warp_epilogue(const MkArgs &a, int kind, int tile, int g, int t,
                                                 const float (&c)[2][4], float (&bv)[2], uint64_t (&bk)[2]) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int m = 2 * t + j;
        const float lo = c[0][j] + c[1][j], hi = c[0][2 + j] + c[1][2 + j];
        if (m >= a.B) continue;
        if (kind == MK_FC) {
            if (tile * 8 + g < a.F) {
                const float u = round_to<__half>(lo);
                const float gt = round_to<__half>(hi);
                const float sig = 1.0f / (1.0f + expf(-gt));
                a.h[(long)m * a.F + tile * 8 + g] = __float2half_rn((gt * sig) * u);
            }
        } else {
            const long lim = (long)(a.V / 8) * 8;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int n = tile * 16 + g + 8 * hh;
                if (n >= a.V) continue;
                const float y = round_to<__half>(hh ? hi : lo);
                if (n < lim && (y > bv[j] || (y == bv[j] && bk[j] != ~0ull))) {
                    const uint64_t k = logits_key(n, 8);
                    if (y > bv[j] || k < bk[j]) {
                        bv[j] = y;
                        bk[j] = k;
                    }
                }
            }
        }
    }
}

// Fused epilogue of one tile; threads 0..127 own (row r, column m).  `red`
// holds the 8 warps' partial tiles; partner rows are summed by the thread in
// the same warp order (bit-identical to the per-op GEMV).
__device__ __forceinline__ float mk_tile_sum(const float *red, int r, int m) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kW; ++w) acc += red[(w * 16 + r) * 8 + m];
    return acc;
}

__device__ void mk_epilogue(const MkArgs &a, const float *red, int kind, int l, int tile, float &best_v,
                            uint64_t &best_k) {
    const int tid = threadIdx.x;
    const int r = (tid >> 3) & 15, m = tid & 7;
    if (tid >= 128 || m >= a.B) return;
    const float acc = mk_tile_sum(red, r, m);
    switch (kind) {
    case MK_QKV: {
        const int nq = a.H * a.D, nk = a.Hk * a.D;
        const int n = tile * 16 + r;
        if (n >= nq + 2 * nk) return;
        const MkLayer &Ly = a.layers[l];
        const float y = round_to<__half>(acc);
        const int pos = a.pos[m];
        const long page = a.block_table[(long)a.seq[m] * a.max_pages + pos / kPg];
        if (n < nq + nk) {
            const float yp = round_to<__half>(mk_tile_sum(red, r ^ 1, m));
            const int dd = (n - (n < nq ? 0 : nq)) % a.D;
            const float *f = a.freqs + (long)pos * a.D + (dd & ~1);
            const float cs = f[0], sn = f[1];
            const float o = (n & 1) ? (yp * sn + y * cs) : (y * cs - yp * sn);
            if (n < nq) {
                a.q[(long)m * nq + n] = __float2half_rn(o);
            } else {
                const int kh = (n - nq) / a.D;
                reinterpret_cast<__half *>(Ly.kpool)[((page * a.Hk + kh) * kPg + pos % kPg) * a.D + dd] =
                    __float2half_rn(o);
            }
        } else {
            const int dd = (n - nq - nk) % a.D, vh = (n - nq - nk) / a.D;
            reinterpret_cast<__half *>(Ly.vpool)[((page * a.Hk + vh) * kPg + pos % kPg) * a.D + dd] =
                __float2half_rn(y);
        }
        break;
    }
    case MK_O:
    case MK_DOWN: {
        const int n = tile * 16 + r;
        if (n >= a.d) return;
        const float y = round_to<__half>(acc);
        __half *xp = a.x + (long)m * a.d + n;
        *xp = __float2half_rn(ldcg_h(xp) + y);
        break;
    }
    case MK_FC: {
        if (r < 8 && tile * 8 + r < a.F) {
            const float u = round_to<__half>(acc);
            const float gt = round_to<__half>(mk_tile_sum(red, r + 8, m));
            const float sig = 1.0f / (1.0f + expf(-gt));
            a.h[(long)m * a.F + tile * 8 + r] = __float2half_rn((gt * sig) * u);
        }
        break;
    }
    default: {  // MK_LOGITS
        const int n = tile * 16 + r;
        if (n >= a.V) return;
        const float y = round_to<__half>(acc);
        const long lim = (long)(a.V / 8) * 8;
        if (n < lim && (y > best_v || (y == best_v && best_k != ~0ull))) {
            const uint64_t k = logits_key(n, 8);
            if (y > best_v || k < best_k) {
                best_v = y;
                best_k = k;
            }
        }
    }
    }
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void sync128() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Causal GQA attention of one (row b, kv head) with the reference's rounding
// points (cuda.cu:767-852, :673-765): warps 0..3, K/V pages through a 4-slot
// cp.async ring in the work area.
template <int D>
__device__ void mk_attention(const MkArgs &a, const Sm &sm, int l, int unit) {
    constexpr int kPageBytes = kPg * D * 2;
    const int b = unit / a.Hk, kvh = unit % a.Hk;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int G = a.H / a.Hk;
    const int Lmax = a.lpad;
    uint8_t *ring = sm.work;                                               // [4][64][D]
    __half *qs = reinterpret_cast<__half *>(ring + kPgSlots * kPageBytes);  // [8][D]
    __half *sc = qs + 8 * D;                                               // [8][lpad]
    float *red = reinterpret_cast<float *>(sc + 8 * Lmax);                 // [8][4]
    const int seq = a.seq[b], pos = a.pos[b];
    const int L = pos + 1;
    const int npages = (L + kPg - 1) / kPg;
    const int Lpad = npages * kPg;
    const int total = 2 * npages;
    const __half *K = reinterpret_cast<const __half *>(a.layers[l].kpool);
    const __half *V = reinterpret_cast<const __half *>(a.layers[l].vpool);
    auto load_page = [&](int i) {
        const int p = i < npages ? i : i - npages;
        const long pg = a.block_table[(long)seq * a.max_pages + p];
        const char *src = reinterpret_cast<const char *>((i < npages ? K : V) + (pg * a.Hk + kvh) * (long)kPg * D);
        char *dst = reinterpret_cast<char *>(ring + (i % kPgSlots) * kPageBytes);
        for (int o = tid * 16; o < kPageBytes; o += 128 * 16) cp_async16(dst + o, src + o);
    };
    for (int i = 0; i < kPgSlots; ++i) {
        if (i < total) load_page(i);
        cp_async_commit();
    }
    const unsigned short *qrow =
        reinterpret_cast<const unsigned short *>(a.q) + (long)b * a.H * D + (long)kvh * G * D;
    for (int i = tid; i < 8 * D; i += 128)
        qs[i] = i < G * D ? __ushort_as_half(__ldcg(qrow + i)) : __float2half_rn(0.f);
    sync128();
    uint32_t qb[D / 16][2];
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
        qb[kk][0] = *reinterpret_cast<const uint32_t *>(qs + g * D + kk * 16 + 2 * t);
        qb[kk][1] = *reinterpret_cast<const uint32_t *>(qs + g * D + kk * 16 + 2 * t + 8);
    }
    const float scale = 1.0f / sqrtf((float)D);
    // ---- pass 1: scores rounded to half, row max per head
    float mx0 = -INFINITY, mx1 = -INFINITY;
    int consumed = 0;
    for (int p = 0; p < npages; ++p, ++consumed) {
        cp_async_wait<kPgSlots - 1>();
        sync128();
        const __half *kt = reinterpret_cast<const __half *>(ring + (consumed % kPgSlots) * kPageBytes) + warp * 16 * D;
        float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
            uint32_t a0, a1, a2, a3;
            ldsm_x4(smem_u32(kt + (lane & 15) * D + kk * 16 + (lane >> 4) * 8), a0, a1, a2, a3);
            mma_f16(c, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
        }
        const int k0 = p * kPg + warp * 16 + g;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int key = k0 + (i >> 1) * 8, hh = 2 * t + (i & 1);
            const float sv = key < L ? round_to<__half>(c[i]) : -INFINITY;
            if (hh < 8) sc[hh * Lmax + key] = __float2half_rn(key < L ? sv : 0.f);
            if (i & 1)
                mx1 = fmaxf(mx1, sv * scale);
            else
                mx0 = fmaxf(mx0, sv * scale);
        }
        sync128();
        if (consumed + kPgSlots < total) load_page(consumed + kPgSlots);
        cp_async_commit();
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
    sync128();
    // ---- softmax numerators (thread -> head hh, keys i0, i0 + 16, ...)
    {
        const int hh = tid >> 4, i0 = tid & 15;
        const float M = fmaxf(fmaxf(red[hh * 4], red[hh * 4 + 1]), fmaxf(red[hh * 4 + 2], red[hh * 4 + 3]));
        float lsum = 0.f;
        for (int j = i0; j < Lpad; j += 16) {
            float e = 0.f;
            if (j < L && hh < G) {
                e = expf(__half2float(sc[hh * Lmax + j]) * scale - M);
                lsum += e;
            }
            sc[hh * Lmax + j] = __float2half_rn(e);
        }
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
        const float inv = 1.0f / lsum;
        for (int j = i0; j < L; j += 16)
            if (hh < G) sc[hh * Lmax + j] = __float2half_rn(__half2float(sc[hh * Lmax + j]) * inv);
    }
    sync128();
    // ---- pass 2: O^T = V^T P^T, warp w owns d-tiles w (and w + 4)
    constexpr int kDT = D / 16;
    constexpr int kNA = kDT > 4 ? 2 : 1;
    float o[kNA][4];
#pragma unroll
    for (int i = 0; i < kNA; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    for (int p = 0; p < npages; ++p, ++consumed) {
        cp_async_wait<kPgSlots - 1>();
        sync128();
        if (p == npages - 1 && L % kPg) {
            // rows past the sequence end hold stale cache bytes; their P is 0, but 0 * NaN is NaN
            __half *vw = reinterpret_cast<__half *>(ring + (consumed % kPgSlots) * kPageBytes);
            const int r0 = L - p * kPg;
            for (int i = tid; i < (kPg - r0) * D; i += 128) vw[r0 * D + i] = __float2half_rn(0.f);
            sync128();
        }
        const __half *vt = reinterpret_cast<const __half *>(ring + (consumed % kPgSlots) * kPageBytes);
#pragma unroll
        for (int ks = 0; ks < kPg / 16; ++ks) {
            const int key0 = p * kPg + ks * 16;
            const uint32_t b0 = *reinterpret_cast<const uint32_t *>(sc + g * Lmax + key0 + 2 * t);
            const uint32_t b1 = *reinterpret_cast<const uint32_t *>(sc + g * Lmax + key0 + 2 * t + 8);
#pragma unroll
            for (int i = 0; i < kNA; ++i) {
                const int d0 = (warp + 4 * i) * 16;
                const int mi = lane >> 3, rr = lane & 7;
                const __half *addr = vt + (ks * 16 + rr + (mi >> 1) * 8) * D + d0 + (mi & 1) * 8;
                uint32_t a0, a1, a2, a3;
                ldsm_x4_t(smem_u32(addr), a0, a1, a2, a3);
                mma_f16(o[i], a0, a1, a2, a3, b0, b1);
            }
        }
        sync128();
        if (consumed + kPgSlots < total) load_page(consumed + kPgSlots);
        cp_async_commit();
    }
    cp_async_wait<0>();
    __half *orow = a.att + (long)b * a.H * D + (long)kvh * G * D;
#pragma unroll
    for (int i = 0; i < kNA; ++i) {
        const int d0 = (warp + 4 * i) * 16;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int dd = d0 + g + (j >> 1) * 8, hh = 2 * t + (j & 1);
            if (hh < G) orow[(long)hh * D + dd] = __float2half_rn(o[i][j]);
        }
    }
    sync128();  // the work area is reused by the next unit
}

// ---------------------------------------------------------------- the kernel
template <int D>
__global__ void __launch_bounds__(kThreads, 1) mk_decode_kernel(const __grid_constant__ MkArgs a, int S) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Sm sm;
    sm.ring = smem_raw;
    sm.bars = reinterpret_cast<uint64_t *>(sm.ring + (size_t)kW * S * kUnit);
    sm.red = reinterpret_cast<float *>(sm.bars + kW * S);
    sm.misc = sm.red + 2 * kW * 16 * 8;
    sm.work = reinterpret_cast<uint8_t *>(sm.misc + 8 + 128 + 2 * 128);
    const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
    const unsigned G = gridDim.x;
    unsigned long long target = a.bar_base;
    int sync_code = 30;

    if (tid < kW * S) mbar_init(sm.bars + tid, 1);
    mbar_fence_init();
    __syncthreads();

    // weights first: they depend on nothing, so the rings fill during the embedding
    Cursor pc;
    pc.gi = 0;
    pc.off = 0;
    pc.offw = 0;
    cur_seek(a, pc, w);
    for (int s = 0; s < S && pc.gi <= 4 * a.L; ++s) {
        if (lane == 0) issue_unit(a, sm, pc, w, S, s);
        cur_next(a, pc, w);
    }

    mk_embed(a);
    grid_sync(a, target += G, sync_code++);

    int consumed = 0, off = 0, offw = 0, ntile_done = 0;
    bool ok = true;
    float best_v = -INFINITY;  // logits winner of this thread (CTA-split logits)
    uint64_t best_k = ~0ull;
    float bv[2] = {-INFINITY, -INFINITY};  // logits winners of this lane's columns (warp-tile logits)
    uint64_t bk[2] = {~0ull, ~0ull};
    bool logits_wm = false;
    auto gemv_phase = [&](int gi, int l, const float *norm) {
        const Gp p = gp_of(a, gi);
        if (norm) mk_stage_norm(a, sm, norm);
        const uint2 *xb;
        long xld;
        bool global_x = false;
        if (p.kind == MK_O) {
            xb = reinterpret_cast<const uint2 *>(a.att);
            xld = (long)a.H * a.D / 4;
            global_x = true;
        } else if (p.kind == MK_DOWN) {
            xb = reinterpret_cast<const uint2 *>(a.h);
            xld = a.F / 4;
            global_x = true;
        } else {
            xb = reinterpret_cast<const uint2 *>(sm.work);
            xld = a.d / 4;
        }
        if (p.wm) {
            const int NW = G * kW;
            for (int tile = first_tile_w(offw, w); tile < p.ntiles; tile += NW) {
                float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
                for (int chunk = 0; chunk < p.nchunks; ++chunk) {
                    const int slot = consumed % S;
                    if (!mbar_wait_bounded(sm.bars + w * S + slot, (consumed / S) & 1, a.err, 21)) ok = false;
                    if (ok) mk_consume<false>(sm.ring + (size_t)(w * S + slot) * kUnit, xb, xld, chunk, a.B, lane, c);
                    __syncwarp();
                    ++consumed;
                    if (pc.gi <= 4 * a.L) {
                        if (lane == 0) issue_unit(a, sm, pc, w, S, slot);
                        cur_next(a, pc, w);
                    }
                }
                mk_warp_epilogue(a, p.kind, tile, lane >> 2, lane & 3, c, bv, bk);
            }
            offw = (offw + p.ntiles) % (int)NW;
            if (p.kind == MK_LOGITS) logits_wm = true;
            return;
        }
        for (int tile = first_tile(off); tile < p.ntiles; tile += G) {
            float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
            for (int chunk = w; chunk < p.nchunks; chunk += kW) {
                const int slot = consumed % S;
                if (!mbar_wait_bounded(sm.bars + w * S + slot, (consumed / S) & 1, a.err, 21)) ok = false;
                if (ok) {
                    const uint8_t *st = sm.ring + (size_t)(w * S + slot) * kUnit;
                    if (global_x)
                        mk_consume<true>(st, xb, xld, chunk, a.B, lane, c);
                    else
                        mk_consume<false>(st, xb, xld, chunk, a.B, lane, c);
                }
                __syncwarp();
                ++consumed;
                if (pc.gi <= 4 * a.L) {
                    if (lane == 0) issue_unit(a, sm, pc, w, S, slot);
                    cur_next(a, pc, w);
                }
            }
            // two partial-tile buffers: tile i + 1 writes the other one, and the
            // barrier of tile i + 1 orders tile i's epilogue reads before tile i + 2's writes
            const int g = lane >> 2, t = lane & 3;
            float *rbuf = sm.red + (ntile_done & 1) * kW * 16 * 8;
            float *red = rbuf + w * 16 * 8;
            red[g * 8 + 2 * t] = c[0][0] + c[1][0];
            red[g * 8 + 2 * t + 1] = c[0][1] + c[1][1];
            red[(g + 8) * 8 + 2 * t] = c[0][2] + c[1][2];
            red[(g + 8) * 8 + 2 * t + 1] = c[0][3] + c[1][3];
            __syncthreads();
            mk_epilogue(a, rbuf, p.kind, l, tile, best_v, best_k);
            ++ntile_done;
        }
        off = (off + p.ntiles) % (int)G;
    };

    for (int l = 0; l < a.L; ++l) {
        const MkLayer &Ly = a.layers[l];
        gemv_phase(4 * l + MK_QKV, l, Ly.attn_norm);
        grid_sync(a, target += G, sync_code++);
        if (w < 4)
            for (int u = blockIdx.x; u < a.B * a.Hk; u += G) mk_attention<D>(a, sm, l, u);
        grid_sync(a, target += G, sync_code++);
        gemv_phase(4 * l + MK_O, l, nullptr);
        grid_sync(a, target += G, sync_code++);
        gemv_phase(4 * l + MK_FC, l, Ly.ffn_norm);
        grid_sync(a, target += G, sync_code++);
        gemv_phase(4 * l + MK_DOWN, l, nullptr);
        grid_sync(a, target += G, sync_code++);
    }
    gemv_phase(4 * a.L, a.L, a.out_norm);

    // per-CTA winner of each row, then CTA 0 picks the token (reference tie order)
    float *sv = sm.misc + 8;
    uint64_t *sk = reinterpret_cast<uint64_t *>(sm.misc + 8 + 128);
    if (logits_wm) {
        // best of the 8 lanes sharing t, then one (value, key) per warp and column
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
        if ((lane >> 2) == 0) {
            sv[w * 8 + 2 * (lane & 3)] = bv[0];
            sk[w * 8 + 2 * (lane & 3)] = bk[0];
            sv[w * 8 + 2 * (lane & 3) + 1] = bv[1];
            sk[w * 8 + 2 * (lane & 3) + 1] = bk[1];
        }
    } else if (tid < 128) {
        sv[tid] = best_v;
        sk[tid] = best_k;
    }
    __syncthreads();
    if (tid < 8) {
        float v = sv[tid];
        uint64_t k = sk[tid];
        for (int r = 1; r < (logits_wm ? kW : 16); ++r) {
            const float ov = sv[r * 8 + tid];
            const uint64_t ok2 = sk[r * 8 + tid];
            if (ov > v || (ov == v && ok2 < k)) {
                v = ov;
                k = ok2;
            }
        }
        a.part_val[(long)blockIdx.x * 8 + tid] = v;
        a.part_key[(long)blockIdx.x * 8 + tid] = k;
    }
    grid_sync(a, target += G, sync_code++);
    if (blockIdx.x == 0 && tid < a.B) {
        float bv = -INFINITY;
        uint64_t bk = ~0ull;
        for (unsigned c = 0; c < G; ++c) {
            const float ov = __ldcg(a.part_val + (long)c * 8 + tid);
            const uint64_t okey = __ldcg(a.part_key + (long)c * 8 + tid);
            if (ov > bv || (ov == bv && okey < bk)) {
                bv = ov;
                bk = okey;
            }
        }
        const int idx = logits_index(bk, 8);
        a.tokens[tid] = idx;
        a.ids[tid] = idx;
        a.pos[tid] += 1;
    }
    (void)ok;
}

template <int D> size_t smem_for(const MkArgs &a, int S) {
    const size_t fixed = (size_t)kW * S * kUnit + (size_t)kW * S * 8 + 2 * kW * 16 * 8 * 4 + (8 + 128 + 256) * 4;
    const size_t xs = (size_t)a.B * a.d * 2;
    const size_t attn = (size_t)kPgSlots * kPg * D * 2 + 8 * D * 2 + (size_t)8 * a.lpad * 2 + 8 * 4 * 4;
    return fixed + (xs > attn ? xs : attn);
}

}  // namespace

size_t mk_smem_bytes(const MkArgs &a, int stages) {
    const size_t s = a.D == 64 ? smem_for<64>(a, stages) : smem_for<128>(a, stages);
    return s <= (size_t)g_rt.max_smem_optin ? s : 0;
}

namespace {
const CUtensorMap *g_loaded_maps = nullptr;  // the maps now in c_maps
}  // namespace

void mk_forget_maps(const CUtensorMap *maps) {
    if (g_loaded_maps == maps) g_loaded_maps = nullptr;
}

cudaError_t mk_launch(const MkArgs &a, int stages, size_t smem, cudaStream_t s) {
    if (4 * a.L + 1 > kMaxMaps) return cudaErrorInvalidValue;
    // the constant bank holds one model's maps: reload when another model launches
    if (g_loaded_maps != a.maps) {
        const cudaError_t e = cudaMemcpyToSymbolAsync(c_maps, a.maps, sizeof(CUtensorMap) * (4 * a.L + 1), 0,
                                                      cudaMemcpyDeviceToDevice, s);
        if (e != cudaSuccess) return e;
        g_loaded_maps = a.maps;
    }
    auto kern = a.D == 64 ? mk_decode_kernel<64> : mk_decode_kernel<128>;
    static size_t configured[2] = {0, 0};
    size_t &cf = configured[a.D == 64 ? 0 : 1];
    if (smem > cf) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        cf = smem;
    }
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorCooperativeLaunchTooLarge;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(g_rt.num_sms);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a, stages);
}

}  // namespace wk
