// Shared definitions of the B200 (sm_100a) wukong op library.
//
// The library sits behind the reference's flat C ABI (cuda.h of liuy/wukong) and
// an extended wk_* API.  It deliberately avoids the C++ runtime library (no
// new/delete, no STL containers, no exceptions) so that the static archive links
// with exactly the cgo line of llm/array.go:4
// (-lcublasLt -lcudart -lm -lcublas).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

namespace wk {

// GGML dtype ids (the reference's wukong.h:15-52 enum, llm/array.go:23-61).
enum DType : int {
    kF32 = 0,
    kF16 = 1,
    kQ4_0 = 2,
    kQ8_0 = 8,
    kBF16 = 30,
    kDTypeCount = 36,
};

struct DTypeInfo {
    const char *name;
    int block_size;
    int type_size;
};
extern const DTypeInfo kDTypes[kDTypeCount];

// Q8_0 block: fp16 scale followed by 32 int8 quants, 34 bytes, no padding.
constexpr int kQ8Block = 32;
constexpr int kQ8Bytes = 34;
// GGUF Q4_0 block: fp16 scale d, then 16 bytes; byte i holds value i (low
// nibble) and value i + 16 (high nibble), each stored as q + 8 (q in [-8, 7]).
constexpr int kQ4Bytes = 18;
// Row bytes of a [rows, K] weight of a GGUF dtype this library streams.
__host__ __device__ inline long quant_row_bytes(int wtype, int K) {
    return wtype == kQ8_0 ? (long)(K / 32) * kQ8Bytes : wtype == kQ4_0 ? (long)(K / 32) * kQ4Bytes
                                                                       : (long)K * (wtype == kF32 ? 4 : 2);
}

// Activation element type that the reference instantiates for a weight dtype:
// float for F32, bf16 for BF16, half for F16 and every quantised type
// (cuda.cu:1324-1338).
inline int act_of(int wtype) { return wtype == kF32 ? kF32 : (wtype == kBF16 ? kBF16 : kF16); }
inline size_t act_size(int act) { return act == kF32 ? 4 : 2; }

// ---------------------------------------------------------------- errors
[[noreturn]] void panic_impl(const char *file, int line, const char *func, const char *fmt, ...);
#define WK_PANIC(...) ::wk::panic_impl(__FILE__, __LINE__, __func__, __VA_ARGS__)
#define WK_CHECK(call)                                                                          \
    do {                                                                                        \
        cudaError_t e_ = (call);                                                                \
        if (e_ != cudaSuccess) WK_PANIC("CUDA error (%d): %s", (int)e_, cudaGetErrorString(e_)); \
    } while (0)
#define WK_CHECK_LAUNCH() WK_CHECK(cudaGetLastError())

// ---------------------------------------------------------------- runtime state
struct Runtime {
    int device = -1;
    int num_sms = 0;
    int max_smem_optin = 0;
    int smem_per_sm = 0;
    cudaStream_t stream = nullptr;
    // device-side error word (mapped pinned memory): bounded waits that give up
    // set a code here
    int *d_error = nullptr;
    int *h_error = nullptr;
    // grow-only scratch arena for op temporaries (stream ordered on `stream`)
    void *ws = nullptr;
    size_t ws_size = 0;
    bool pdl = true;      // programmatic dependent launch on the hot kernels
    bool tc_gemm = true;  // tcgen05 GEMM for activation blocks of >= 16 rows
    int warp_tile_min = 4096;  // SwiGLU / logits layers with this many 16-row tiles run one tile per warp
    long l2_prefetch_max = 12L << 20;  // engine: bytes of the next layer's weights each linear layer prefetches into L2
    // limit of the cross-GPU flag waits of the tensor-parallel exchange
    // (WUKONG_WAIT_LIMIT_MS, default one second)
    unsigned long long wait_limit_ns = 1000000000ull;
    // called by cuda_fini with the device index (set by parts that cache
    // per-device state; a pointer, so cuda.h's objects do not link them in)
    void (*on_fini)(int device) = nullptr;
    // split-K workspace of the tcgen05 GEMM (all launches are ordered on `stream`)
    float *splitk_ws = nullptr;
    size_t splitk_ws_floats = 0;
    int *splitk_counter = nullptr;
    int splitk_tiles = 0;
};
extern Runtime g_rt;

void ensure_init();
// Scratch memory valid until the next call that asks for scratch.
void *scratch(size_t bytes);
inline cudaStream_t stream() { return g_rt.stream; }
void set_device_current();
void check_device_error();

// ---------------------------------------------------------------- device helpers
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

template <typename T> struct Act;
template <> struct Act<float> {
    static __device__ __forceinline__ float load(const float *p) { return *p; }
    static __device__ __forceinline__ float to_f(float v) { return v; }
    static __device__ __forceinline__ float from_f(float v) { return v; }
    static __device__ __forceinline__ float round(float v) { return v; }
};
template <> struct Act<__half> {
    static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
    static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
    static __device__ __forceinline__ float round(float v) { return __half2float(__float2half_rn(v)); }
};
template <> struct Act<__nv_bfloat16> {
    static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
    static __device__ __forceinline__ float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
};

__device__ __forceinline__ float to_float(float v) { return v; }
__device__ __forceinline__ float to_float(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> __device__ __forceinline__ T from_float(float v);
template <> __device__ __forceinline__ float from_float<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_float<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float v) {
    return __float2bfloat16_rn(v);
}
template <typename T> __device__ __forceinline__ float round_to(float v) { return to_float(from_float<T>(v)); }

// ---------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait: gives up after one second (far above any legitimate wait for a
// bulk copy), records `code` in the device error word and returns false.  The
// caller keeps its control flow uniform so that no other warp is left waiting.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, int *err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        for (int i = 0; i < 64; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > 1000000000ull) break;
    }
    if (err) atomicCAS(err, 0, code);
    return false;
}
// System-scope flag store / load for flags that other GPUs read or write.
__device__ __forceinline__ void st_release_sys(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// Wait until *flag >= e; false (code recorded in the error word) after limit_ns.
__device__ __forceinline__ bool wait_flag(const unsigned long long *flag, unsigned long long e, int *err, int code,
                                          unsigned long long limit_ns) {
    if (ld_acquire_sys(flag) >= e) return true;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys(flag) < e) {
        if (globaltimer_ns() - t0 > limit_ns) {
            if (err) atomicCAS(err, 0, code);
            return false;
        }
        __nanosleep(32);
    }
    return true;
}

// Prefetch this CTA's share of [base, base + bytes) into L2 (fire and forget):
// the weights of the next kernel in a decode step stream from DRAM while the
// current kernel is still running.
__device__ __forceinline__ void l2_prefetch_slice(const void *base, long bytes, int part, int parts) {
    const long per = ((bytes + parts - 1) / parts + 15) & ~15L;
    long lo = (long)part * per, hi = lo + per < bytes ? lo + per : bytes;
    hi &= ~15L;
    const char *p = (const char *)base;
    for (long o = lo; o < hi; o += 262144) {
        const long n = hi - o < 262144 ? hi - o : 262144;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p + o), "r"((uint32_t)n) : "memory");
    }
}

// 1-D bulk copy global -> shared, completing on `bar` (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void bulk_g2s_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ void mma_f16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Four int8 quants (one 32-bit word, bytes q0..q3) -> two half2 {q0,q1},{q2,q3},
// exact: byte b is placed as the mantissa of 1024 + (b ^ 0x80), then 1152 is
// subtracted (all values are integers below 2048, so no rounding occurs).
__device__ __forceinline__ void i8x4_to_h2x2(uint32_t w, __half2 &lo, __half2 &hi) {
    const uint32_t x = w ^ 0x80808080u;
    uint32_t l = __byte_perm(x, 0x64646464u, 0x5140);  // {0x64, b1, 0x64, b0}
    uint32_t h = __byte_perm(x, 0x64646464u, 0x5342);  // {0x64, b3, 0x64, b2}
    const __half2 bias = __half2half2(__ushort_as_half((unsigned short)0x6480));  // 1152.0
    lo = __hsub2(*reinterpret_cast<__half2 *>(&l), bias);
    hi = __hsub2(*reinterpret_cast<__half2 *>(&h), bias);
}
__device__ __forceinline__ uint32_t h2_as_u32(__half2 v) { return *reinterpret_cast<uint32_t *>(&v); }
// Four 4-bit fields (one per byte of n, each 0..15, the stored q + 8) -> two
// half2 {q0,q1},{q2,q3}, exact: 1024 + n as the mantissa, minus 1032.
__device__ __forceinline__ void u4x4_to_h2x2(uint32_t n, __half2 &lo, __half2 &hi) {
    uint32_t l = __byte_perm(n, 0x64646464u, 0x5140);
    uint32_t h = __byte_perm(n, 0x64646464u, 0x5342);
    const __half2 bias = __half2half2(__ushort_as_half((unsigned short)0x6408));  // 1032.0
    lo = __hsub2(*reinterpret_cast<__half2 *>(&l), bias);
    hi = __hsub2(*reinterpret_cast<__half2 *>(&h), bias);
}

// Argmax order of the reference's argmax kernel (cuda.cu:480-531) as a sort key:
// element idx of a row is read by thread (idx / pack) % 256 in iteration
// (idx / pack) / 256 as the (idx % pack)-th value of a packed load; ties go to the
// first iteration within a thread, then to the lane / warp with the smaller
// bit-reversed index (the shfl_down tree).  Smaller key = preferred on ties.
__device__ __forceinline__ uint64_t logits_key(long idx, int pack) {
    const long p = idx / pack;
    const uint32_t tid = (uint32_t)(p & 255), j = (uint32_t)(p >> 8), e = (uint32_t)(idx - p * pack);
    const uint32_t bw = __brev(tid >> 5) >> 27, bl = __brev(tid & 31) >> 27;
    return ((uint64_t)bw << 58) | ((uint64_t)bl << 53) | ((uint64_t)j << 8) | e;
}
// Inverse of logits_key (-1 for the empty key ~0).
__device__ __forceinline__ int logits_index(uint64_t key, int pack) {
    if (key == ~0ull) return -1;
    const uint32_t bw = (uint32_t)(key >> 58) & 31, bl = (uint32_t)(key >> 53) & 31;
    const uint32_t tid8 = ((__brev(bw) >> 27) << 5) | (__brev(bl) >> 27);
    const long j = (long)((key >> 8) & ((1ull << 45) - 1));
    return (int)(((j << 8) + tid8) * pack + (int)(key & 255));
}

// One Q8_0 block (32 k, two MMA k-slices) of rows g and g + 8 of the staged tile:
// lane t takes quant bytes 4t..4t+3 of each 16-value half.  Odd blocks start
// their quants 4-byte aligned (34 * odd + 2 = 0 mod 4); even ones are realigned
// by a byte permute of two neighbouring words.
__device__ __forceinline__ void q8_block(const uint8_t *r0, const uint8_t *r1, int off, bool odd, int t, uint2 x0,
                                         uint2 x1, float (&c)[2][4]) {
    const __half2 s0 = __half2half2(*reinterpret_cast<const __half *>(r0 + off));
    const __half2 s1 = __half2half2(*reinterpret_cast<const __half *>(r1 + off));
    uint32_t q0[2], q1[2];  // [slice] quant words for rows g, g+8
    if (odd) {
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
        const uint2 xv = h ? x1 : x0;
        mma_f16(c[h], a0, a1, a2, a3, xv.x, xv.y);
    }
}

// One Q4_0 block (32 k, two MMA k-slices) of rows g and g + 8 of the staged
// tile: lane t takes quant bytes 4t..4t+3 (values 4t..4t+3 of the first
// 16-slice in their low nibbles, of the second in their high nibbles).  Odd
// blocks start their quants 4-byte aligned (18 * odd + 2 = 0 mod 4).
__device__ __forceinline__ void q4_block(const uint8_t *r0, const uint8_t *r1, int off, bool odd, int t, uint2 x0,
                                         uint2 x1, float (&c)[2][4]) {
    const __half2 s0 = __half2half2(*reinterpret_cast<const __half *>(r0 + off));
    const __half2 s1 = __half2half2(*reinterpret_cast<const __half *>(r1 + off));
    uint32_t w0, w1;
    if (odd) {
        w0 = *reinterpret_cast<const uint32_t *>(r0 + off + 2 + 4 * t);
        w1 = *reinterpret_cast<const uint32_t *>(r1 + off + 2 + 4 * t);
    } else {
        const uint32_t *p0 = reinterpret_cast<const uint32_t *>(r0 + off + 4 * t);
        const uint32_t *p1 = reinterpret_cast<const uint32_t *>(r1 + off + 4 * t);
        w0 = __byte_perm(p0[0], p0[1], 0x5432);
        w1 = __byte_perm(p1[0], p1[1], 0x5432);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint32_t n0 = h ? (w0 >> 4) & 0x0F0F0F0Fu : w0 & 0x0F0F0F0Fu;
        const uint32_t n1 = h ? (w1 >> 4) & 0x0F0F0F0Fu : w1 & 0x0F0F0F0Fu;
        __half2 lo0, hi0, lo1, hi1;
        u4x4_to_h2x2(n0, lo0, hi0);
        u4x4_to_h2x2(n1, lo1, hi1);
        const uint32_t a0 = h2_as_u32(__hmul2(lo0, s0)), a2 = h2_as_u32(__hmul2(hi0, s0));
        const uint32_t a1 = h2_as_u32(__hmul2(lo1, s1)), a3 = h2_as_u32(__hmul2(hi1, s1));
        const uint2 xv = h ? x1 : x0;
        mma_f16(c[h], a0, a1, a2, a3, xv.x, xv.y);
    }
}

// ldmatrix: four 8x8 b16 tiles (optionally transposed) from shared memory
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

}  // namespace wk
