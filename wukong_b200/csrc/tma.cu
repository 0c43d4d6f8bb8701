// Host side of TMA: tensor-map encoding and a per-weight map cache.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "wukong_internal.cuh"

namespace wk {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
    if (!g_encode) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        WK_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !fn) WK_PANIC("cuTensorMapEncodeTiled is not available");
        g_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
    }
    return g_encode;
}

struct MapEntry {
    const void *w;
    long rows, row_bytes;
    int box_inner, box_rows;
    unsigned long long stamp;
    CUtensorMap map;
};
constexpr int kMapCache = 4096;
MapEntry *g_maps = nullptr;
unsigned long long g_stamp = 0;

}  // namespace

bool encode_map_2d(CUtensorMap *m, const void *base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
                   uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_stride_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encoder()(m, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

const CUtensorMap *weight_map(const void *w, long rows, long row_bytes, int box_inner, int box_rows) {
    if (((uintptr_t)w % 16) || (row_bytes % 16) || rows <= 0) return nullptr;
    if (!g_maps) g_maps = (MapEntry *)calloc(kMapCache, sizeof(MapEntry));
    int victim = 0;
    for (int i = 0; i < kMapCache; ++i) {
        MapEntry &e = g_maps[i];
        if (e.w == w && e.rows == rows && e.row_bytes == row_bytes && e.box_inner == box_inner &&
            e.box_rows == box_rows) {
            e.stamp = ++g_stamp;
            return &e.map;
        }
        if (e.stamp < g_maps[victim].stamp) victim = i;
    }
    MapEntry &e = g_maps[victim];
    if (!encode_map_2d(&e.map, w, CU_TENSOR_MAP_DATA_TYPE_UINT16, (uint64_t)row_bytes / 2, (uint64_t)rows,
                       (uint64_t)row_bytes, (uint32_t)box_inner, (uint32_t)box_rows, CU_TENSOR_MAP_SWIZZLE_NONE)) {
        e.w = nullptr;
        e.stamp = 0;
        return nullptr;
    }
    e.w = w;
    e.rows = rows;
    e.row_bytes = row_bytes;
    e.box_inner = box_inner;
    e.box_rows = box_rows;
    e.stamp = ++g_stamp;
    return &e.map;
}

void forget_weight_maps(const void *w) {
    if (!g_maps) return;
    for (int i = 0; i < kMapCache; ++i)
        if (g_maps[i].w == w) {
            g_maps[i].w = nullptr;
            g_maps[i].stamp = 0;
        }
}

}  // namespace wk
