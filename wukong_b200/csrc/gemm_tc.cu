// tcgen05 / TMEM GEMM with the Q8_0 dequantisation fused into the A-operand
// load, for prefill and batched decode (activation rows M >= 16).
//
//   D[128 weight rows x BN tokens] (fp32, TMEM) = W_tile[128 x K] . X_tile[BN x K]^T
//
// Reference semantics (cuda.cu:1095-1111, :270-341): W is dequantised to half
// exactly as the reference does (w = (half)(float(scale) * q)), multiplied with
// half activations, accumulated in fp32 and rounded once to half at the store.
//
// CTA = 10 warps, one output tile per CTA:
//   warp 0 (lane 0)  TMA producer: raw Q8_0 tiles (128 rows x 256 k = 128 x 272 B,
//                    one 2-D box) and activation tiles (BN rows x 64 k, 128-byte
//                    swizzle); for 16-bit weights also the A tiles.
//   warp 1           allocates TMEM; lane 0 issues tcgen05.mma (M=128, N=BN,
//                    K=16 per instruction) and tcgen05.commit.
//   warps 2..9       two threads per weight row (warps 2..5 Q8_0 blocks 0..3 of
//                    each 256-k raw stage, warps 6..9 blocks 4..7): read the raw
//                    bytes from shared memory (16-byte loads), dequantise in
//                    registers (byte-permute -> exact half2, half2 multiply by the
//                    scale) and write the 128-byte-swizzled fp16 A tile the UMMA
//                    descriptor expects; after the K loop warps 2..5 drain TMEM
//                    (tcgen05.ld) and run the fused epilogue (store+bias,
//                    residual, RoPE+KV append, SwiGLU pairing of up/gate rows).
// The operand ring holds 4 stages for 128-token tiles and 6 for 64 / 32.
// Every mbarrier wait is bounded (one second); a wait that gives up records an
// error code and the CTA runs to completion without further waiting.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "wukong_internal.cuh"

namespace wk {

namespace {

constexpr int kThreads = 320;
constexpr int kMaxSlots = 6;                    // 64-k operand stages (deepest ring)
// operand ring depth: 4 stages of 128-token B tiles fit beside the raw ring, 6 of 64 / 32
template <int BN> struct Slots {
    static constexpr int n = BN >= 256 ? 3 : (BN >= 128 ? 4 : 6);
};
constexpr int kRawSlots = 2;                    // 256-k raw Q8_0 stages
constexpr int kATileBytes = 128 * 128;          // 128 rows x 64 halves
constexpr int kRawBytes = 128 * 272;            // 128 rows x 8 Q8_0 blocks
constexpr int kKB = 256;                        // k per raw stage

// ---------------------------------------------------------------- PTX
__device__ __forceinline__ void tma2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"((uint64_t)map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// UMMA shared-memory descriptor: K-major operand in the canonical 128-byte
// swizzle layout (rows of 128 bytes, 8-row groups 1024 bytes apart).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);  // start address
    d |= (uint64_t)1 << 16;                             // leading byte offset (unused for this layout)
    d |= (uint64_t)(1024 >> 4) << 32;                   // stride byte offset: next 8-row group
    d |= (uint64_t)1 << 46;                             // descriptor version
    d |= (uint64_t)2 << 61;                             // 128-byte swizzle
    return d;
}

struct Bars {
    uint64_t raw_full[kRawSlots], raw_empty[kRawSlots];
    uint64_t a_full[kMaxSlots], b_full[kMaxSlots], ab_empty[kMaxSlots];
    uint64_t acc_full;
    uint32_t tmem;
};

template <int BN> struct Layout {
    static constexpr int kBTile = BN * 128;
    static constexpr size_t kA = 0;
    static constexpr size_t kB = kA + (size_t)Slots<BN>::n * kATileBytes;
    static constexpr size_t kRaw = kB + (size_t)Slots<BN>::n * kBTile;
    static constexpr size_t kBars = kRaw + (size_t)kRawSlots * kRawBytes;
    static constexpr size_t kTotal = kBars + sizeof(Bars) + 1024;  // + alignment slack
};

// Dequantise 64 k (Q8_0 blocks 2j, 2j+1 of this row's 272 raw bytes; `w` holds
// the row's bytes [BASE, BASE + 4 NW)) into the 128-byte swizzled A row.
template <int BASE, int NW>
__device__ __forceinline__ void dequant_sub(const uint32_t (&w)[NW], int j, uint8_t *arow, int row) {
#pragma unroll
    for (int bb = 0; bb < 2; ++bb) {
        const int b = 2 * j + bb;  // compile-time after unrolling j
        const int off = 34 * b;    // byte offset of the block
        // scale: bytes off, off+1
        const uint32_t sw = w[(off - BASE) >> 2];
        const uint32_t sbits = (off & 2) ? (sw >> 16) : (sw & 0xffffu);
        const __half2 s2 = __half2half2(__ushort_as_half((unsigned short)sbits));
        // 32 quants start at off + 2: 8 words, realigned when off + 2 is not 4-aligned
        uint32_t q[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int byte = off + 2 + 4 * i;
            if (byte & 2)
                q[i] = __byte_perm(w[(byte - BASE) >> 2], w[((byte - BASE) >> 2) + 1], 0x5432);
            else
                q[i] = w[(byte - BASE) >> 2];
        }
        // 32 halves = 4 x 16-byte chunks (chunk c covers k = 8c .. 8c+7 of the 64-k sub-tile)
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
            __half2 h[4];
            i8x4_to_h2x2(q[2 * cc], h[0], h[1]);
            i8x4_to_h2x2(q[2 * cc + 1], h[2], h[3]);
            uint4 v;
            v.x = h2_as_u32(__hmul2(h[0], s2));
            v.y = h2_as_u32(__hmul2(h[1], s2));
            v.z = h2_as_u32(__hmul2(h[2], s2));
            v.w = h2_as_u32(__hmul2(h[3], s2));
            const int c = bb * 4 + cc;
            *reinterpret_cast<uint4 *>(arow + ((c ^ (row & 7)) << 4)) = v;
        }
    }
}

template <typename T>
__device__ __forceinline__ void store_out(const GemmArgs &a, int n, int m, float acc, const float *partner) {
    // partner: value of the paired row (RoPE: n ^ 1, SwiGLU: the gate row)
    switch (a.epi) {
    case EPI_STORE: {
        if (a.bias) acc += to_float(reinterpret_cast<const T *>(a.bias)[n]);
        reinterpret_cast<T *>(a.out)[(long)m * a.ldo + n] = from_float<T>(acc);
        break;
    }
    case EPI_PARTIAL: {
        reinterpret_cast<float *>(a.out)[(long)m * a.ldo + n] = acc;
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
            const float yp = round_to<T>(*partner);
            const int dd = (n - (n < a.nq ? 0 : a.nq)) % a.hd;
            const float *f = a.freqs + (long)pos * a.hd + (dd & ~1);
            const float cs = f[0], sn = f[1];
            const float o = (n & 1) ? (yp * sn + y * cs) : (y * cs - yp * sn);
            if (n < a.nq) {
                reinterpret_cast<T *>(a.out)[(long)m * a.ldo + n] = from_float<T>(o);
            } else {
                const int kh = (n - a.nq) / a.hd;
                const long page = a.block_table[(long)a.seq[m] * a.max_pages + pos / a.page];
                reinterpret_cast<T *>(a.kpool)[((page * a.kv_heads + kh) * a.page + pos % a.page) * a.hd + dd] =
                    from_float<T>(o);
            }
        } else {
            const int dd = (n - a.nq - a.nk) % a.hd, vh = (n - a.nq - a.nk) / a.hd;
            const long page = a.block_table[(long)a.seq[m] * a.max_pages + pos / a.page];
            reinterpret_cast<T *>(a.vpool)[((page * a.kv_heads + vh) * a.page + pos % a.page) * a.hd + dd] =
                from_float<T>(y);
        }
        break;
    }
    case EPI_SWIGLU: {
        const float u = round_to<T>(acc);
        const float g = round_to<T>(*partner);
        const float sig = 1.0f / (1.0f + expf(-g));
        reinterpret_cast<T *>(a.out)[(long)m * a.ldo + n] = from_float<T>((g * sig) * u);
        break;
    }
    default:
        break;
    }
}

// Vectorised epilogue of 8 consecutive output rows n..n+7 (a 16-byte group)
// for one token m: the same formulas and rounding points as store_out.
template <typename T>
__device__ __forceinline__ void store_out8(const GemmArgs &a, int n, int m, const float (&v)[8], const float *gate) {
    switch (a.epi) {
    case EPI_STORE: {
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = v[j];
        if (a.bias) {
            const uint4 b = *reinterpret_cast<const uint4 *>(reinterpret_cast<const T *>(a.bias) + n);
            const T *bt = reinterpret_cast<const T *>(&b);
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] += to_float(bt[j]);
        }
        uint4 u;
        T *ut = reinterpret_cast<T *>(&u);
#pragma unroll
        for (int j = 0; j < 8; ++j) ut[j] = from_float<T>(o[j]);
        *reinterpret_cast<uint4 *>(reinterpret_cast<T *>(a.out) + (long)m * a.ldo + n) = u;
        break;
    }
    case EPI_PARTIAL: {
        float4 *o = reinterpret_cast<float4 *>(reinterpret_cast<float *>(a.out) + (long)m * a.ldo + n);
        o[0] = make_float4(v[0], v[1], v[2], v[3]);
        o[1] = make_float4(v[4], v[5], v[6], v[7]);
        break;
    }
    case EPI_RESID: {
        const uint4 r = *reinterpret_cast<const uint4 *>(reinterpret_cast<const T *>(a.res) + (long)m * a.ldr + n);
        const T *rt = reinterpret_cast<const T *>(&r);
        uint4 u;
        T *ut = reinterpret_cast<T *>(&u);
#pragma unroll
        for (int j = 0; j < 8; ++j) ut[j] = from_float<T>(to_float(rt[j]) + round_to<T>(v[j]));
        *reinterpret_cast<uint4 *>(reinterpret_cast<T *>(a.out) + (long)m * a.ldo + n) = u;
        break;
    }
    case EPI_QKV: {
        const int pos = a.pos[m];
        uint4 u;
        T *ut = reinterpret_cast<T *>(&u);
        const bool rope = n < a.nq + a.nk;
        const int base = n < a.nq ? 0 : (rope ? a.nq : a.nq + a.nk);
        const int dd = (n - base) % a.hd;  // group start within its head (the 8 rows share the head)
        if (rope) {
            const float *f = a.freqs + (long)pos * a.hd + dd;
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
                const float y0 = round_to<T>(v[j]), y1 = round_to<T>(v[j + 1]);
                const float cs = f[j], sn = f[j + 1];
                ut[j] = from_float<T>(y0 * cs - y1 * sn);
                ut[j + 1] = from_float<T>(y0 * sn + y1 * cs);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) ut[j] = from_float<T>(v[j]);
        }
        if (n < a.nq) {
            *reinterpret_cast<uint4 *>(reinterpret_cast<T *>(a.out) + (long)m * a.ldo + n) = u;
        } else {
            const int h = (n - base) / a.hd;
            const long page = a.block_table[(long)a.seq[m] * a.max_pages + pos / a.page];
            T *pool = reinterpret_cast<T *>(rope ? a.kpool : a.vpool);
            *reinterpret_cast<uint4 *>(pool + ((page * a.kv_heads + h) * a.page + pos % a.page) * a.hd + dd) = u;
        }
        break;
    }
    case EPI_SWIGLU: {
        uint4 u;
        T *ut = reinterpret_cast<T *>(&u);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float up = round_to<T>(v[j]);
            const float g = round_to<T>(gate[j]);
            const float sig = 1.0f / (1.0f + expf(-g));
            ut[j] = from_float<T>((g * sig) * up);
        }
        *reinterpret_cast<uint4 *>(reinterpret_cast<T *>(a.out) + (long)m * a.ldo + n) = u;
        break;
    }
    default:
        break;
    }
}

template <typename T, int WT, int BN>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const __grid_constant__ GemmArgs a) {
    using L = Layout<BN>;
    constexpr int kASlots = Slots<BN>::n;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled tiles
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *A = smem + L::kA;
    uint8_t *B = smem + L::kB;
    uint8_t *RAW = smem + L::kRaw;
    Bars *bars = reinterpret_cast<Bars *>(smem + L::kBars);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_tile = blockIdx.x, m0 = blockIdx.y * BN;
    const bool swiglu = a.epi == EPI_SWIGLU;
    // split-K (gridDim.z > 1): this CTA's K range [kz0, kz0 + K / gridDim.z)
    const int Kc = a.K / (int)gridDim.z;
    const int kz0 = (int)blockIdx.z * Kc;
    const int nkb = Kc / kKB;       // raw stages (Q8_0) / 4 x 64-k subs
    const int nsub = Kc / 64;       // operand stages
    const int kb0 = kz0 / kKB, ks0 = kz0 / 64;
    constexpr bool kQ8 = WT == kQ8_0;
    constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;
    constexpr uint32_t kIdesc = (1u << 4) | ((WT == kBF16 ? 1u : 0u) << 7) | ((WT == kBF16 ? 1u : 0u) << 10) |
                                ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);

    if (threadIdx.x == 0) {
        for (int i = 0; i < kRawSlots; ++i) {
            mbar_init(&bars->raw_full[i], 1);
            mbar_init(&bars->raw_empty[i], 256);  // every dequantising thread
        }
        for (int i = 0; i < kASlots; ++i) {
            mbar_init(&bars->a_full[i], kQ8 ? 128 : 1);
            mbar_init(&bars->b_full[i], 1);
            mbar_init(&bars->ab_empty[i], 1);
        }
        mbar_init(&bars->acc_full, 1);
        mbar_fence_init();
    }
    if (warp == 1) tc_alloc(&bars->tmem, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem;
    int *err = a.err;
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {
            // weights do not depend on the previous kernel: start them first
            const int wy = swiglu ? n_tile * 64 : n_tile * 128;
            auto issue_raw = [&](int kb) {
                const int s = kb % kRawSlots;
                mbar_expect_tx(&bars->raw_full[s], kRawBytes);
                if (swiglu) {
                    tma2d(RAW + (size_t)s * kRawBytes, &a.wmap, (kb0 + kb) * 136, wy, &bars->raw_full[s]);
                    tma2d(RAW + (size_t)s * kRawBytes + 64 * 272, &a.wmap, (kb0 + kb) * 136, a.F + wy,
                          &bars->raw_full[s]);
                } else {
                    tma2d(RAW + (size_t)s * kRawBytes, &a.wmap, (kb0 + kb) * 136, wy, &bars->raw_full[s]);
                }
            };
            int raw_issued = 0;
            if (kQ8)
                for (; raw_issued < kRawSlots && raw_issued < nkb; ++raw_issued) issue_raw(raw_issued);
            pdl_wait();
            for (int i = 0; i < nsub && ok; ++i) {
                const int s = i % kASlots;
                if (i >= kASlots && !mbar_wait_bounded(&bars->ab_empty[s], ((i / kASlots) - 1) & 1, err, 10)) {
                    ok = false;
                    break;
                }
                const uint32_t tx = (uint32_t)(L::kBTile + (kQ8 ? 0 : kATileBytes));
                mbar_expect_tx(&bars->b_full[s], tx);
                tma2d(B + (size_t)s * L::kBTile, &a.xmap, (ks0 + i) * 64, m0, &bars->b_full[s]);
                if (!kQ8) {
                    if (swiglu) {
                        tma2d(A + (size_t)s * kATileBytes, &a.wmap, (ks0 + i) * 64, wy, &bars->b_full[s]);
                        tma2d(A + (size_t)s * kATileBytes + 64 * 128, &a.wmap, (ks0 + i) * 64, a.F + wy,
                              &bars->b_full[s]);
                    } else {
                        tma2d(A + (size_t)s * kATileBytes, &a.wmap, (ks0 + i) * 64, wy, &bars->b_full[s]);
                    }
                }
                // keep the raw ring one stage ahead of the operand stages
                if (kQ8 && (i % 4) == 3 && raw_issued < nkb) {
                    const int kb = raw_issued;
                    if (!mbar_wait_bounded(&bars->raw_empty[kb % kRawSlots], ((kb / kRawSlots) - 1) & 1, err, 11)) {
                        ok = false;
                        break;
                    }
                    issue_raw(kb);
                    ++raw_issued;
                }
            }
        }
        pdl_trigger();
    } else if (warp == 1) {
        if (lane == 0) {
            pdl_wait();
            for (int i = 0; i < nsub && ok; ++i) {
                const int s = i % kASlots;
                const uint32_t par = (i / kASlots) & 1;
                if (!mbar_wait_bounded(&bars->b_full[s], par, err, 12)) ok = false;
                if (kQ8 && ok && !mbar_wait_bounded(&bars->a_full[s], par, err, 13)) ok = false;
                if (!ok) break;
                tc_fence_after();
                const uint32_t abase = smem_u32(A + (size_t)s * kATileBytes);
                const uint32_t bbase = smem_u32(B + (size_t)s * L::kBTile);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    tc_mma(tmem, sw128_desc(abase + 32 * kk), sw128_desc(bbase + 32 * kk), kIdesc, (i | kk) != 0);
                tc_commit(&bars->ab_empty[s]);
            }
            tc_commit(&bars->acc_full);
        }
        pdl_trigger();
    } else {
        // warps 2..9 dequantise: row = (warp % 4) * 32 + lane (the TMEM lane quarter
        // of warps 2..5, which also run the epilogue); warps 2..5 take Q8_0 blocks
        // 0..3 of each 256-k raw stage (A sub-tiles 0, 1), warps 6..9 blocks 4..7
        const int row = (warp & 3) * 32 + lane;
        const int half = (warp - 2) >> 2;
        pdl_trigger();
        if (kQ8) {
            for (int kb = 0; kb < nkb && ok; ++kb) {
                const int rs = kb % kRawSlots;
                if (!mbar_wait_bounded(&bars->raw_full[rs], (kb / kRawSlots) & 1, err, 14)) {
                    ok = false;
                    break;
                }
                // bytes [128 half, 128 half + 144) of the row: blocks 4 half .. 4 half + 3
                uint32_t w[36];
                const uint4 *src =
                    reinterpret_cast<const uint4 *>(RAW + (size_t)rs * kRawBytes + row * 272 + half * 128);
#pragma unroll
                for (int i = 0; i < 9; ++i) {
                    const uint4 v = src[i];
                    w[4 * i] = v.x;
                    w[4 * i + 1] = v.y;
                    w[4 * i + 2] = v.z;
                    w[4 * i + 3] = v.w;
                }
                mbar_arrive(&bars->raw_empty[rs]);  // this part of the raw row is in registers
#pragma unroll
                for (int jj = 0; jj < 2; ++jj) {
                    const int j = 2 * half + jj;
                    const int i = kb * 4 + j;
                    const int s = i % kASlots;
                    if (i >= kASlots && !mbar_wait_bounded(&bars->ab_empty[s], ((i / kASlots) - 1) & 1, err, 15)) {
                        ok = false;
                        break;
                    }
                    uint8_t *arow = A + (size_t)s * kATileBytes + row * 128;
                    if (half == 0)
                        dequant_sub<0>(w, jj, arow, row);
                    else
                        dequant_sub<128>(w, 2 + jj, arow, row);
                    fence_proxy_async();  // generic-proxy writes -> visible to tcgen05.mma
                    mbar_arrive(&bars->a_full[s]);
                }
            }
        }
        if (half == 0) {
        // epilogue: TMEM -> registers -> fused store (reads residual / positions
        // written by earlier kernels)
        pdl_wait();
        const bool acc_ok = ok && mbar_wait_bounded(&bars->acc_full, 0, err, 16);
        tc_fence_after();
        float *xchg = reinterpret_cast<float *>(RAW);  // [128 rows][32 columns] for row pairing
        // split-K: every split stores its fp32 tile ([128 rows][BN] per split and
        // tile); the last split of the tile to arrive adds them in split order
        // (the same sum whatever the arrival order) and runs the epilogue
        const int nz = (int)gridDim.z;
        const long tile_id = (long)blockIdx.y * gridDim.x + blockIdx.x;
        bool run_epi = true;
        if (nz > 1) {
            float *mine = a.ws + ((tile_id * nz + blockIdx.z) * 128 + row) * BN;
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t v[32];
                tc_ld32(tmem + (((uint32_t)(warp & 3) * 32) << 16) + (uint32_t)c0, v);
#pragma unroll
                for (int i = 0; i < 32; i += 4)
                    *reinterpret_cast<float4 *>(mine + c0 + i) =
                        acc_ok ? make_float4(__uint_as_float(v[i]), __uint_as_float(v[i + 1]),
                                             __uint_as_float(v[i + 2]), __uint_as_float(v[i + 3]))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            __threadfence();
            asm volatile("bar.sync 1, 128;" ::: "memory");
            __shared__ int s_last;
            if (threadIdx.x == 64) s_last = atomicAdd(a.ws_counter + tile_id, 1) == nz - 1;
            asm volatile("bar.sync 1, 128;" ::: "memory");
            run_epi = s_last != 0;
            if (run_epi) __threadfence();
        }
        // the tile's accumulators for 32 tokens from c0: TMEM, or the splits' sum
        auto load_acc = [&](int c0, uint32_t (&v)[32]) {
            if (nz == 1) {
                tc_ld32(tmem + (((uint32_t)(warp & 3) * 32) << 16) + (uint32_t)c0, v);
                if (!acc_ok)
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = 0u;
                return;
            }
            float acc[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) acc[i] = 0.f;
            for (int z = 0; z < nz; ++z) {
                const float4 *src = reinterpret_cast<const float4 *>(a.ws + ((tile_id * nz + z) * 128 + row) * BN + c0);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float4 f = __ldcg(src + i);
                    acc[4 * i] += f.x;
                    acc[4 * i + 1] += f.y;
                    acc[4 * i + 2] += f.z;
                    acc[4 * i + 3] += f.w;
                }
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(acc[i]);
        };
        if (run_epi && a.vec) {
            // the accumulators of 32 tokens go through shared memory ([32 tokens][128 rows]
            // fp32) so that each thread then handles 16-byte groups of 8 consecutive outputs
            float *st = reinterpret_cast<float *>(RAW);
            const int te = threadIdx.x - 64;  // 0..127 over warps 2..5
            const int groups = swiglu ? 8 : 16;  // 8-row groups per token (SwiGLU: the 64 up rows)
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t v[32];
                load_acc(c0, v);
                asm volatile("bar.sync 1, 128;" ::: "memory");  // the previous chunk's groups are done
#pragma unroll
                for (int i = 0; i < 32; ++i) st[i * 128 + row] = __uint_as_float(v[i]);
                asm volatile("bar.sync 1, 128;" ::: "memory");
                for (int it = te; it < 32 * groups; it += 128) {
                    const int i = it / groups, r0 = (it % groups) * 8;
                    const int m = m0 + c0 + i;
                    const int n = swiglu ? n_tile * 64 + r0 : n_tile * 128 + r0;
                    if (m >= a.M || n >= (swiglu ? a.F : a.N)) continue;
                    float vv[8], gg[8];
                    const float4 *src = reinterpret_cast<const float4 *>(st + i * 128 + r0);
                    const float4 x0 = src[0], x1 = src[1];
                    vv[0] = x0.x, vv[1] = x0.y, vv[2] = x0.z, vv[3] = x0.w;
                    vv[4] = x1.x, vv[5] = x1.y, vv[6] = x1.z, vv[7] = x1.w;
                    if (swiglu) {
                        const float4 *gs = reinterpret_cast<const float4 *>(st + i * 128 + 64 + r0);
                        const float4 y0 = gs[0], y1 = gs[1];
                        gg[0] = y0.x, gg[1] = y0.y, gg[2] = y0.z, gg[3] = y0.w;
                        gg[4] = y1.x, gg[5] = y1.y, gg[6] = y1.z, gg[7] = y1.w;
                    }
                    store_out8<T>(a, n, m, vv, gg);
                }
            }
        }
        for (int c0 = 0; run_epi && !a.vec && c0 < BN; c0 += 32) {
            uint32_t v[32];
            load_acc(c0, v);
            // pairing partner (RoPE: row ^ 1 in the neighbouring lane; SwiGLU: row + 64)
            if (swiglu) {
                asm volatile("bar.sync 1, 128;" ::: "memory");
#pragma unroll
                for (int i = 0; i < 32; ++i) xchg[row * 33 + i] = __uint_as_float(v[i]);
                asm volatile("bar.sync 1, 128;" ::: "memory");
            }
            const int n = swiglu ? (n_tile * 64 + row) : (n_tile * 128 + row);
            const bool row_ok = swiglu ? (row < 64 && n < a.F) : (n < a.N);
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int m = m0 + c0 + i;
                float pv = 0.f;
                if (a.epi == EPI_QKV) pv = __shfl_xor_sync(0xffffffffu, __uint_as_float(v[i]), 1);
                if (swiglu && row < 64) pv = xchg[(row + 64) * 33 + i];
                if (row_ok && m < a.M) store_out<T>(a, n, m, __uint_as_float(v[i]), &pv);
            }
        }
        if (nz > 1 && run_epi && threadIdx.x == 64) a.ws_counter[tile_id] = 0;  // ready for the next launch
        }  // half == 0: the epilogue warps
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tc_dealloc(tmem, kTmemCols);
    }
}

template <typename T, int WT, int BN> void launch_tc(const GemmArgs &a, cudaStream_t s, bool pdl) {
    auto kern = gemm_tc_kernel<T, WT, BN>;
    const size_t smem = Layout<BN>::kTotal;
    static bool configured = false;
    if (!configured) {
        WK_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        configured = true;
    }
    const int ntiles = a.epi == EPI_SWIGLU ? (a.F + 63) / 64 : (a.N + 127) / 128;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ntiles, (a.M + BN - 1) / BN, a.ksplit);
    cfg.blockDim = dim3(kThreads);
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

bool gemm_tc_supported(int wtype, int act, int K, int N, int epi, int F) {
    if (act == kF32) return false;
    if (wtype == kQ8_0 && (act != kF16 || K % kKB)) return false;
    if ((wtype == kF16 && act != kF16) || (wtype == kBF16 && act != kBF16)) return false;
    if (wtype != kQ8_0 && wtype != kF16 && wtype != kBF16) return false;
    if (K % 64) return false;
    if (epi == EPI_SWIGLU && F % 64) return false;
    if (epi == EPI_LOGITS) return false;
    (void)N;
    return true;
}

void gemm_tc(GemmArgs a, int act, cudaStream_t s) {
    if (!gemm_tc_supported(a.wtype, act, a.K, a.N, a.epi, a.F)) WK_PANIC("gemm_tc: unsupported problem");
    if (!a.err) a.err = g_rt.d_error;
    const size_t es = 2;
    // activations: [M rows][K] with row stride ldx, boxes of 64 k x BN rows, 128-byte swizzle
    // token tile: 64 for M >= 48 so that M = 128 spreads over twice the CTAs
    // 256-token tiles for long blocks (half the operand traffic per FLOP of 128-token
    // tiles: the main loop is bound by operand loads, not by the tensor core)
    const int BN = a.M >= 1024 ? 256 : a.M >= 256 ? 128 : (a.M >= 48 ? 64 : 32);
    if (((uintptr_t)a.x % 16) || ((a.ldx * es) % 16)) WK_PANIC("gemm_tc: activations must be 16-byte aligned rows");
    if (!encode_map_2d(&a.xmap, a.x, act == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                       (uint64_t)a.K, (uint64_t)a.M, (uint64_t)a.ldx * es, 64, (uint32_t)BN,
                       CU_TENSOR_MAP_SWIZZLE_128B))
        WK_PANIC("gemm_tc: activation tensor map");
    const long rows = a.epi == EPI_SWIGLU ? 2L * a.F : (long)a.N;
    const int box_rows = a.epi == EPI_SWIGLU ? 64 : 128;
    if (a.wtype == kQ8_0) {
        const CUtensorMap *m = weight_map(a.w, rows, (long)(a.K / 32) * 34, 136, box_rows);
        if (!m) WK_PANIC("gemm_tc: weight rows are not 16-byte aligned");
        a.wmap = *m;
    } else {
        if (((uintptr_t)a.w % 16) || !encode_map_2d(&a.wmap, a.w,
                                                     a.wtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                                                     (uint64_t)a.K, (uint64_t)rows, (uint64_t)a.K * 2, 64,
                                                     (uint32_t)box_rows, CU_TENSOR_MAP_SWIZZLE_128B))
            WK_PANIC("gemm_tc: weight tensor map");
    }
    // 16-byte groups of outputs when every row the epilogue touches is 16-byte aligned
    auto al16 = [](const void *p, long ld, size_t esz) {
        return p == nullptr || (((uintptr_t)p % 16) == 0 && ((size_t)ld * esz) % 16 == 0);
    };
    a.vec = (a.epi == EPI_SWIGLU ? a.F % 8 == 0 : a.N % 8 == 0) &&
            al16(a.out, a.ldo, a.epi == EPI_PARTIAL ? 4 : es) && (a.epi != EPI_RESID || al16(a.res, a.ldr, es)) &&
            (a.epi != EPI_STORE || al16(a.bias, 0, es)) &&
            (a.epi != EPI_QKV || (a.hd % 8 == 0 && a.nq % 8 == 0 && a.nk % 8 == 0 && al16(a.kpool, 0, es) &&
                                  al16(a.vpool, 0, es)));
    // split-K when the output tiles would leave most SMs idle (small batches):
    // up to one CTA per SM, each K slice a multiple of 256
    a.ksplit = 1;
    {
        const long tiles = (long)(a.epi == EPI_SWIGLU ? (a.F + 63) / 64 : (a.N + 127) / 128) * ((a.M + BN - 1) / BN);
        if (BN <= 64 && g_rt.splitk_ws && tiles * 2 <= g_rt.num_sms) {
            int z = (int)(g_rt.num_sms / tiles);
            while (z > 1 && (a.K % (z * kKB) || (size_t)tiles * z * 128 * BN > g_rt.splitk_ws_floats ||
                             tiles > g_rt.splitk_tiles))
                --z;
            a.ksplit = z;
        }
        a.ws = g_rt.splitk_ws;
        a.ws_counter = g_rt.splitk_counter;
    }
    const bool pdl = g_rt.pdl && a.pdl;
#define WK_TC_LAUNCH(T, W)                        \
    do {                                          \
        if (BN == 256)                            \
            launch_tc<T, W, 256>(a, s, pdl);      \
        else if (BN == 128)                       \
            launch_tc<T, W, 128>(a, s, pdl);      \
        else if (BN == 64)                        \
            launch_tc<T, W, 64>(a, s, pdl);       \
        else                                      \
            launch_tc<T, W, 32>(a, s, pdl);       \
    } while (0)
    if (a.wtype == kQ8_0)
        WK_TC_LAUNCH(__half, kQ8_0);
    else if (a.wtype == kF16)
        WK_TC_LAUNCH(__half, kF16);
    else
        WK_TC_LAUNCH(__nv_bfloat16, kBF16);
#undef WK_TC_LAUNCH
}

}  // namespace wk
