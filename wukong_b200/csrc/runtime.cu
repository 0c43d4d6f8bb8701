// Device, stream and memory entry points of the C ABI (cuda.h:1-6, :17).
//
// Reference semantics (cuda.cu:1017-1082, :1267-1275): one device, one stream,
// stream-ordered allocation, host->device copies asynchronous, device->host
// copies synchronous.  Errors abort the process with a message, as the
// reference's panic macro does (wukong.h:173-188).
#include <stdarg.h>
#include <stdlib.h>

#include "common.cuh"
#include "wukong_internal.cuh"

namespace wk {

const DTypeInfo kDTypes[kDTypeCount] = {
    {"F32", 1, 4},          {"F16", 1, 2},         {"GGML_TYPE_Q4_0", 32, 18}, {"GGML_TYPE_Q4_1", 32, 20},
    {"GGML_TYPE_Q4_2", 32, 20}, {"GGML_TYPE_Q4_3", 32, 20}, {"GGML_TYPE_Q5_0", 32, 22}, {"GGML_TYPE_Q5_1", 32, 24},
    {"GGML_TYPE_Q8_0", 32, 34}, {"GGML_TYPE_Q8_1", 32, 40}, {"GGML_TYPE_Q2_K", 256, 84}, {"GGML_TYPE_Q3_K", 256, 110},
    {"GGML_TYPE_Q4_K", 256, 144}, {"GGML_TYPE_Q5_K", 256, 176}, {"GGML_TYPE_Q6_K", 256, 210},
    {"GGML_TYPE_Q8_K", 256, 292}, {"GGML_TYPE_IQ2_XXS", 256, 66}, {"GGML_TYPE_IQ2_XS", 256, 74},
    {"GGML_TYPE_IQ3_XXS", 256, 98}, {"GGML_TYPE_IQ1_S", 256, 50}, {"GGML_TYPE_IQ4_NL", 32, 18},
    {"GGML_TYPE_IQ3_S", 256, 110}, {"GGML_TYPE_IQ2_S", 256, 82}, {"GGML_TYPE_IQ4_XS", 256, 136},
    {"Int8", 1, 1},         {"Int16", 1, 2},       {"Int32", 1, 4},            {"Int64", 1, 8},
    {"F64", 1, 8},          {"GGML_TYPE_IQ1_M", 256, 56}, {"BF16", 1, 2},      {"GGML_TYPE_Q4_0_4_4", 32, 18},
    {"GGML_TYPE_Q4_0_4_8", 32, 18}, {"GGML_TYPE_Q4_0_8_8", 32, 18}, {"GGML_TYPE_TQ1_0", 256, 54},
    {"GGML_TYPE_TQ2_0", 256, 66},
};

Runtime g_rt;

void panic_impl(const char *file, int line, const char *func, const char *fmt, ...) {
    fprintf(stderr, "%s:%d:%s(): ", file, line, func);
    va_list ap;
    va_start(ap, fmt);
    vfprintf(stderr, fmt, ap);
    va_end(ap);
    fprintf(stderr, "\n");
    fflush(stderr);
    exit(EXIT_FAILURE);
}

void check_device_error() {
    int err = g_rt.h_error ? *(volatile int *)g_rt.h_error : 0;
    if (err) WK_PANIC("a device-side bounded wait gave up (code %d)", err);
}

void set_device_current() {
    if (g_rt.device >= 0) WK_CHECK(cudaSetDevice(g_rt.device));
}

void ensure_init() {
    if (g_rt.device < 0) WK_PANIC("cuda_init() has not been called");
    set_device_current();
}

void *scratch(size_t bytes) {
    bytes = (bytes + 255) & ~(size_t)255;
    if (bytes > g_rt.ws_size) {
        if (g_rt.ws) WK_CHECK(cudaFreeAsync(g_rt.ws, g_rt.stream));
        size_t sz = bytes + bytes / 4;
        WK_CHECK(cudaMallocAsync(&g_rt.ws, sz, g_rt.stream));
        g_rt.ws_size = sz;
    }
    return g_rt.ws;
}

}  // namespace wk

using namespace wk;

extern "C" {

// cuda.cu:1017-1049
void cuda_init(int idx) {
    srand(0);
    g_rt.device = idx;
    WK_CHECK(cudaSetDevice(idx));
    WK_CHECK(cudaStreamCreateWithFlags(&g_rt.stream, cudaStreamNonBlocking));
    cudaDeviceProp prop;
    WK_CHECK(cudaGetDeviceProperties(&prop, idx));
    g_rt.num_sms = prop.multiProcessorCount;
    g_rt.max_smem_optin = (int)prop.sharedMemPerBlockOptin;
    g_rt.smem_per_sm = (int)prop.sharedMemPerMultiprocessor;
    if (prop.major < 10) WK_PANIC("this library is built for sm_100a (B200); device %d is sm_%d%d", idx, prop.major, prop.minor);
    // error word in mapped pinned memory: kernels write it, the host reads it
    // after any synchronisation without an extra copy
    WK_CHECK(cudaHostAlloc((void **)&g_rt.h_error, sizeof(int), cudaHostAllocMapped));
    *g_rt.h_error = 0;
    WK_CHECK(cudaHostGetDevicePointer((void **)&g_rt.d_error, g_rt.h_error, 0));
    const char *pdl = getenv("WUKONG_PDL");
    g_rt.pdl = !(pdl && pdl[0] == '0');
    const char *tc = getenv("WUKONG_TC_GEMM");
    g_rt.tc_gemm = !(tc && tc[0] == '0');
    const char *wt = getenv("WUKONG_WARP_TILE_MIN");
    if (wt && atoi(wt) > 0) g_rt.warp_tile_min = atoi(wt);
    const char *pfm = getenv("WUKONG_L2_PREFETCH_MB");
    if (pfm && atoi(pfm) >= 0) g_rt.l2_prefetch_max = (long)atoi(pfm) << 20;
    const char *wl = getenv("WUKONG_WAIT_LIMIT_MS");
    if (wl && atoi(wl) > 0) g_rt.wait_limit_ns = 1000000ull * (unsigned long long)atoi(wl);
    // split-K partials of the tcgen05 GEMM: at most 2 CTAs per SM of 128 x 64 fp32 tiles
    g_rt.splitk_tiles = 1024;
    g_rt.splitk_ws_floats = (size_t)2 * g_rt.num_sms * 128 * 64;
    WK_CHECK(cudaMalloc(&g_rt.splitk_ws, sizeof(float) * g_rt.splitk_ws_floats));
    WK_CHECK(cudaMalloc(&g_rt.splitk_counter, sizeof(int) * g_rt.splitk_tiles));
    WK_CHECK(cudaMemset(g_rt.splitk_counter, 0, sizeof(int) * g_rt.splitk_tiles));
    printf("Running on GPU %d: %s, Compute Capability %d.%d\n", idx, prop.name, prop.major, prop.minor);
    fflush(stdout);
    layers_init();
}

// cuda.cu:1051-1057
void cuda_fini(void) {
    if (g_rt.device < 0) return;
    set_device_current();
    layers_fini();
    WK_CHECK(cudaStreamSynchronize(g_rt.stream));
    if (g_rt.on_fini) g_rt.on_fini(g_rt.device);
    if (g_rt.ws) WK_CHECK(cudaFree(g_rt.ws));
    if (g_rt.splitk_ws) WK_CHECK(cudaFree(g_rt.splitk_ws));
    if (g_rt.splitk_counter) WK_CHECK(cudaFree(g_rt.splitk_counter));
    g_rt.splitk_ws = nullptr;
    g_rt.splitk_counter = nullptr;
    g_rt.ws = nullptr;
    g_rt.ws_size = 0;
    WK_CHECK(cudaFreeHost(g_rt.h_error));
    g_rt.h_error = nullptr;
    g_rt.d_error = nullptr;
    WK_CHECK(cudaStreamDestroy(g_rt.stream));
    g_rt.stream = nullptr;
    g_rt.device = -1;
}

// cuda.cu:1060-1065
void *cuda_malloc(size_t size) {
    ensure_init();
    void *p = nullptr;
    WK_CHECK(cudaMallocAsync(&p, size, g_rt.stream));
    return p;
}

// cuda.cu:1067-1070
void cuda_free(void *ptr) {
    if (!ptr) return;
    ensure_init();
    prefix_cache_forget(ptr);
    forget_weight_maps(ptr);
    WK_CHECK(cudaFreeAsync(ptr, g_rt.stream));
}

// cuda.cu:1072-1075
void cuda_to_device(void *dst, void *src, size_t size) {
    ensure_init();
    prefix_cache_note_upload(dst, src, size);
    WK_CHECK(cudaMemcpyAsync(dst, src, size, cudaMemcpyHostToDevice, g_rt.stream));
}

// cuda.cu:1077-1082
void cuda_to_host(void *dst, void *src, size_t size) {
    ensure_init();
    WK_CHECK(cudaMemcpyAsync(dst, src, size, cudaMemcpyDeviceToHost, g_rt.stream));
    WK_CHECK(cudaStreamSynchronize(g_rt.stream));
    check_device_error();
}

int wk_device_error(int clear) {
    if (g_rt.device < 0 || !g_rt.h_error) return 0;
    set_device_current();
    WK_CHECK(cudaStreamSynchronize(g_rt.stream));
    const int e = *(volatile int *)g_rt.h_error;
    if (clear) *(volatile int *)g_rt.h_error = 0;
    return e;
}

// cuda.cu:1267-1275: row concatenation of two tensors of the same dtype.
void cuda_cat(void *out, const void *a, const void *b, int arow, int brow, int col, int dtype) {
    ensure_init();
    if (dtype < 0 || dtype >= kDTypeCount) WK_PANIC("Unsupported dtype: %d", dtype);
    const DTypeInfo &info = kDTypes[dtype];
    size_t asize = (size_t)arow * col * info.type_size / info.block_size;
    size_t bsize = (size_t)brow * col * info.type_size / info.block_size;
    prefix_cache_note_write(out, asize + bsize);
    WK_CHECK(cudaMemcpyAsync(out, a, asize, cudaMemcpyDeviceToDevice, g_rt.stream));
    WK_CHECK(cudaMemcpyAsync((char *)out + asize, b, bsize, cudaMemcpyDeviceToDevice, g_rt.stream));
}

}  // extern "C"
