// Tensor parallelism inside one node, one process per GPU (Megatron-style):
// column-parallel q|k|v and up|gate, row-parallel o and down (each rank holds a
// K-slice and produces fp32 partial sums), vocabulary-parallel logits.
//
// Exchanges per layer: one all-reduce of the fp32 partials after o and one
// after down ([rows, d] fp32), followed by the residual add with the
// reference's rounding (y = T(sum of partials), x = T(x + y): the same formula
// as the single-GPU RESID epilogue, cuda.cu:423-435 after :1095-1111, up to
// the fp32 summation order).  The logits head exchanges one (value, order key)
// winner per row and rank and picks the best with the reference argmax's tie
// order (cuda.cu:480-531), so the token equals the single-GPU token.
//
// The collectives are NCCL's, loaded at run time (dlopen of libnccl.so.2) so
// that the library still links with the reference's cgo line
// (-lcublasLt -lcudart -lm -lcublas) and hosts without NCCL are unaffected.
#include <dlfcn.h>
#include <nccl.h>  // types only; every function is resolved with dlsym
#include <string.h>

#include "common.cuh"
#include "wukong_ext.h"
#include "wukong_internal.cuh"

namespace wk {

namespace {

struct NcclApi {
    void *handle = nullptr;
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
};
NcclApi g_nccl;
ncclComm_t g_comm = nullptr;
int g_rank = 0, g_world = 1;

int load_nccl() {
    if (g_nccl.handle) return 0;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return fail("tensor parallelism needs NCCL: dlopen(libnccl.so.2) failed: %s", dlerror());
    NcclApi a;
    a.handle = h;
#define WK_NCCL_SYM(field, name)                                           \
    a.field = (decltype(a.field))dlsym(h, name);                          \
    if (!a.field) return fail("libnccl.so.2 does not export %s", name);
    WK_NCCL_SYM(get_unique_id, "ncclGetUniqueId")
    WK_NCCL_SYM(comm_init_rank, "ncclCommInitRank")
    WK_NCCL_SYM(comm_destroy, "ncclCommDestroy")
    WK_NCCL_SYM(all_reduce, "ncclAllReduce")
    WK_NCCL_SYM(all_gather, "ncclAllGather")
    WK_NCCL_SYM(error_string, "ncclGetErrorString")
#undef WK_NCCL_SYM
    g_nccl = a;
    return 0;
}

void nccl_check(ncclResult_t r, const char *what) {
    if (r != ncclSuccess) WK_PANIC("%s failed: %s", what, g_nccl.error_string ? g_nccl.error_string(r) : "?");
}

// x = T(x + T(p)): the residual add of a row-parallel layer after its all-reduce
template <typename T> __global__ void resid_from_partial_kernel(T *__restrict__ x, const float *__restrict__ p, long n) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = from_float<T>(to_float(x[i]) + round_to<T>(p[i]));
}

// rec: [world][chunk bytes] with, per rank, keys [B] (u64) then values [B] (f32)
__global__ void argmax_combine_kernel(int *__restrict__ tokens, const uint8_t *__restrict__ rec, long chunk, int B,
                                      int world, int pack) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    float bv = -INFINITY;
    uint64_t bk = ~0ull;
    for (int r = 0; r < world; ++r) {
        const uint64_t k = reinterpret_cast<const uint64_t *>(rec + r * chunk)[b];
        const float v = reinterpret_cast<const float *>(rec + r * chunk + 8L * B)[b];
        if (k == ~0ull) continue;
        if (v > bv || (v == bv && k < bk)) {
            bv = v;
            bk = k;
        }
    }
    tokens[b] = logits_index(bk, pack);
}

}  // namespace

bool tp_active() { return g_comm != nullptr && g_world > 1; }
int tp_rank() { return g_rank; }
int tp_world() { return g_world; }

void tp_allreduce_f32(float *buf, size_t n, cudaStream_t s) {
    nccl_check(g_nccl.all_reduce(buf, buf, n, ncclFloat32, ncclSum, g_comm, s), "ncclAllReduce");
}

size_t tp_winner_chunk(int B) { return ((size_t)B * 12 + 15) / 16 * 16; }

void tp_argmax_combine(int *tokens, const void *send, void *recv, int B, int pack, cudaStream_t s) {
    const size_t chunk = tp_winner_chunk(B);
    nccl_check(g_nccl.all_gather(send, recv, chunk, ncclUint8, g_comm, s), "ncclAllGather");
    argmax_combine_kernel<<<(B + 127) / 128, 128, 0, s>>>(tokens, (const uint8_t *)recv, (long)chunk, B, g_world,
                                                         pack);
    WK_CHECK_LAUNCH();
}

template <typename T> void resid_from_partial(T *x, const float *p, long n, cudaStream_t s) {
    if (n <= 0) return;
    resid_from_partial_kernel<T><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(x, p, n);
    WK_CHECK_LAUNCH();
}
template void resid_from_partial<__half>(__half *, const float *, long, cudaStream_t);
template void resid_from_partial<__nv_bfloat16>(__nv_bfloat16 *, const float *, long, cudaStream_t);

}  // namespace wk

using namespace wk;

extern "C" {

int wk_tp_unique_id(void *id) {
    if (!id) return fail("wk_tp_unique_id: null buffer");
    if (load_nccl()) return -1;
    ncclUniqueId u;
    ncclResult_t r = g_nccl.get_unique_id(&u);
    if (r != ncclSuccess) return fail("ncclGetUniqueId: %s", g_nccl.error_string(r));
    memcpy(id, &u, sizeof(u));
    return 0;
}

int wk_tp_init(int rank, int world, const void *id) {
    if (world < 1 || rank < 0 || rank >= world || !id) return fail("wk_tp_init: bad rank %d / world %d", rank, world);
    if (g_rt.device < 0) return fail("wk_tp_init: cuda_init() has not been called");
    if (g_comm) return fail("wk_tp_init: already initialised (call wk_tp_fini first)");
    if (load_nccl()) return -1;
    set_device_current();
    ncclUniqueId u;
    memcpy(&u, id, sizeof(u));
    ncclResult_t r = g_nccl.comm_init_rank(&g_comm, world, u, rank);
    if (r != ncclSuccess) {
        g_comm = nullptr;
        return fail("ncclCommInitRank(rank %d of %d): %s", rank, world, g_nccl.error_string(r));
    }
    g_rank = rank;
    g_world = world;
    return 0;
}

void wk_tp_fini(void) {
    if (g_comm) {
        cudaStreamSynchronize(stream());
        g_nccl.comm_destroy(g_comm);
    }
    g_comm = nullptr;
    g_rank = 0;
    g_world = 1;
}

int wk_tp_rank(void) { return g_rank; }
int wk_tp_world(void) { return g_world; }

}  // extern "C"
