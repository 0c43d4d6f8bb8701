// wk_predict_noalloc: greedy next-token ids like cuda_predict, with no device
// memory allocation.
//
// Who needs it: hosts that have already handed the whole GPU to their own
// memory manager (a serving process that reserves every free byte of HBM for
// its KV-cache pool at start-up, so a later cudaMalloc fails), and hosts on a
// latency-critical loop where cudaMalloc / cudaFree would synchronise the
// device and stall every stream.  cuda_predict draws its argmax partials from
// buffers that cuda_init allocates and, on its non-fused paths, allocates a
// logits buffer per call; this variant keeps all of its scratch in one
// fixed-size array that is part of the library image.
//
// The kernel is the same dequant-fused logits GEMV that cuda_predict runs
// (gemv.cu, EPI_LOGITS): each CTA writes one argmax partial per activation
// row, and the last CTA to finish (an atomic counter) reduces them to token
// ids in the reference kernel's tie order (cuda.cu:1416-1428).
//
// Scratch: g_predict_scratch below, 8 passes x (512 CTAs x 8 rows) partials
// (fp32 value + 64-bit order key) and one counter per pass: 393,472 bytes,
// held by every GPU that loads this library until the process exits.  One
// pass covers 8 sequences, so a call takes at most kMaxBatch = 64 sequences.
// Every call shares the array; two calls that overlap on the GPU (different
// streams, or threads racing on the library stream) corrupt each other's
// partials.  Calls on the library stream run one after another and are safe.
// Each call clears the per-pass counters before its first pass; the partials
// need no clearing (every pass writes the ones it reads).
//
// Set-up: cuda_init() must have run (it creates the library stream at
// start-up).  The first call on each device looks up the array's device
// address with cudaGetSymbolAddress, which can also load this library's GPU
// code onto the device; make that first call before any stream capture.
// This entry point does not end a pass of the opt-in prefix cache
// (WUKONG_PREFIX_CACHE=1), which allocates its own KV pages and so is for
// hosts that can allocate.
#include <atomic>

#include "common.cuh"
#include "wukong_ext.h"
#include "wukong_internal.cuh"

namespace wk {

namespace {

constexpr int kPassRows = 8;                     // activation rows per GEMV pass
constexpr int kMaxBatch = 64;                    // sequences per call
constexpr int kPasses = kMaxBatch / kPassRows;   // 8
constexpr int kMaxCol = 32768;                   // model width: the normalised row stays in shared memory
constexpr size_t kPartials = (size_t)kMaxLogitCtas * kPassRows;  // per pass
constexpr size_t kValOff = 0;
constexpr size_t kKeyOff = kValOff + sizeof(float) * kPartials * kPasses;                // 131072
constexpr size_t kCountOff = kKeyOff + sizeof(unsigned long long) * kPartials * kPasses;  // 393216
constexpr size_t kScratchBytes = kCountOff + 256;                                         // 393472
static_assert(kKeyOff % 256 == 0 && kCountOff % 256 == 0, "scratch regions stay 256-byte aligned");

// The scratch itself.  In host code this name is only a stand-in for the
// device variable; the host passes kernels the address that
// cudaGetSymbolAddress returns for the current device.
static __device__ __align__(256) unsigned char g_predict_scratch[kScratchBytes];

// The per-pass counters must start at zero (the last CTA of each pass resets
// its own, but a call that stopped early may have left one behind).
__global__ void clear_counters_kernel(int passes) {
    int *counter = reinterpret_cast<int *>(g_predict_scratch + kCountOff);
    if ((int)threadIdx.x < passes) counter[threadIdx.x] = 0;
}

constexpr int kMaxDevices = 64;
std::atomic<unsigned char *> g_scratch_addr[kMaxDevices];

// cuda_fini drops the cached address: after a new cuda_init (which may follow a
// reset of the device's context) the first call looks it up again.
void forget_address(int device) {
    if (device >= 0 && device < kMaxDevices) g_scratch_addr[device].store(nullptr, std::memory_order_release);
}

// Device address of g_predict_scratch on the current device, looked up once
// per device (the first call on each device does it).
unsigned char *scratch_address(int device) {
    unsigned char *p = g_scratch_addr[device].load(std::memory_order_acquire);
    if (p) return p;
    void *addr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&addr, g_predict_scratch);
    if (e != cudaSuccess || !addr) {
        fail("wk_predict_noalloc: cudaGetSymbolAddress of the scratch array failed on device %d: %s", device,
             cudaGetErrorString(e));
        return nullptr;
    }
    g_scratch_addr[device].store((unsigned char *)addr, std::memory_order_release);
    g_rt.on_fini = forget_address;
    return (unsigned char *)addr;
}

}  // namespace

}  // namespace wk

using namespace wk;

extern "C" {

int wk_predict_noalloc(int *out, const void *ff, const void *norm_weight, const void *out_weight, int batch, int row,
                       int col, int wsize, float eps, int dtype) {
    if (g_rt.device < 0) return fail("wk_predict_noalloc: cuda_init() has not been called");
    if (g_rt.device >= kMaxDevices) return fail("wk_predict_noalloc: device %d >= %d", g_rt.device, kMaxDevices);
    if (batch < 1 || batch > kMaxBatch)
        return fail("wk_predict_noalloc: batch %d outside [1, %d] (the static scratch holds %d sequences per call)",
                    batch, kMaxBatch, kMaxBatch);
    if (row < 1 || wsize < 1) return fail("wk_predict_noalloc: row %d / wsize %d must be positive", row, wsize);
    if (!out || !ff || !norm_weight || !out_weight) return fail("wk_predict_noalloc: null tensor argument");
    if (dtype != kF16 && dtype != kBF16 && dtype != kQ8_0)
        return fail("wk_predict_noalloc: dtype %d not supported (F16, BF16 or Q8_0 output weights)", dtype);
    const int act = act_of(dtype);
    if (!gemv_supported(dtype, act, col))
        return fail("wk_predict_noalloc: col %d must be a multiple of %d for this dtype", col, dtype == kQ8_0 ? 32 : 16);
    if (col > kMaxCol) return fail("wk_predict_noalloc: col %d > %d", col, kMaxCol);
    if ((uintptr_t)ff % 8) return fail("wk_predict_noalloc: ff must be 8-byte aligned");
    cudaError_t e = cudaSetDevice(g_rt.device);
    if (e != cudaSuccess) return fail("wk_predict_noalloc: cudaSetDevice: %s", cudaGetErrorString(e));
    unsigned char *base = scratch_address(g_rt.device);
    if (!base) return -1;

    cudaStream_t s = stream();
    const int passes = (batch + kPassRows - 1) / kPassRows;
    clear_counters_kernel<<<1, 32, 0, s>>>(passes);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail("wk_predict_noalloc: launch: %s", cudaGetErrorString(e));
    float *val = reinterpret_cast<float *>(base + kValOff);
    unsigned long long *key = reinterpret_cast<unsigned long long *>(base + kKeyOff);
    int *counter = reinterpret_cast<int *>(base + kCountOff);
    const size_t es = act_size(act);
    for (int p = 0; p < passes; ++p) {
        const int m0 = p * kPassRows;
        GemvArgs a;
        a.w = (const uint8_t *)out_weight;
        a.wtype = dtype;
        a.N = wsize;
        a.K = col;
        // last row of each sequence: ff[b, row - 1, :]
        a.x = (const char *)ff + ((size_t)m0 * row + (row - 1)) * col * es;
        a.ldx = (long)row * col;
        a.M = batch - m0 < kPassRows ? batch - m0 : kPassRows;
        a.norm_w = (const float *)norm_weight;
        a.eps = eps;
        a.epi = EPI_LOGITS;
        a.out = nullptr;
        a.part_val = val + (size_t)p * kPartials;
        a.part_key = key + (size_t)p * kPartials;
        a.counter = counter + p;
        a.tokens = out + m0;
        a.pack = 16 / (int)es;
        gemv(a, act, s);
    }
    return 0;
}

}  // extern "C"
