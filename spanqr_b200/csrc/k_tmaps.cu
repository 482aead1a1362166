// Per-matrix TMA tensor maps of the row-major X and Q of every matrix in a call (2-D fp32; tiles of 32 columns x 128
// rows for the solve, 128 columns x 32 rows for the Gram; rows past K and columns past r read as zeros).  The host encodes one template per operand (cuTensorMapEncodeTiled, fetched from
// the driver at run time); k_tmaps copies it once per matrix into the workspace and patches in that matrix's address
// with tensormap.replace, so batched calls whose pointers live only on the device get maps too.
#include <cudaTypedefs.h>

#include <mutex>

#include "kernels.h"

namespace spq {

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

cudaError_t encoder() {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    return g_encode ? cudaSuccess : cudaErrorNotSupported;
}
}  // namespace

cudaError_t encode_rows(CUtensorMap* m, const void* base, int rows, int cols, long long ld, int box_cols, int box_rows) {
    cudaError_t e = encoder();
    if (e != cudaSuccess) return e;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * sizeof(float)};
    const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, es,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

struct TmapTemplates {
    CUtensorMap m[TMAPS_PER_MATRIX];
};

__global__ void k_tmaps(PtrArg p, int B, const __grid_constant__ TmapTemplates t, char* __restrict__ maps) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    const MatPtr mp = p.tab ? p.tab[b] : p.one;
    int4* d = reinterpret_cast<int4*>(maps + (size_t)b * TMAPS_PER_MATRIX * 128);
    const int4* src = reinterpret_cast<const int4*>(&t);
#pragma unroll
    for (int i = 0; i < 8 * TMAPS_PER_MATRIX; ++i) d[i] = src[i];
#pragma unroll
    for (int m = 0; m < TMAPS_PER_MATRIX; ++m) {
        const void* a = (m == TMAP_X || m == TMAP_GX) ? static_cast<const void*>(mp.X) : static_cast<const void*>(mp.Q);
        asm volatile("tensormap.replace.tile.global_address.global.b1024.b64 [%0], %1;" ::"l"(d + 8 * m), "l"(a)
                     : "memory");
    }
    asm volatile("fence.proxy.tensormap::generic.release.gpu;" ::: "memory");
}

cudaError_t launch_tmaps(PtrArg p, int K, int r, long long ldx, long long ldq, int B, const void* any, char* maps,
                         cudaStream_t st) {
    alignas(64) TmapTemplates t;
    cudaError_t e = encode_rows(&t.m[TMAP_X], any, K, r, ldx, TMAP_BOX_COLS, TMAP_BOX_ROWS);
    if (e == cudaSuccess) e = encode_rows(&t.m[TMAP_Q], any, K, r, ldq, TMAP_BOX_COLS, TMAP_BOX_ROWS);
    if (e == cudaSuccess) e = encode_rows(&t.m[TMAP_GX], any, K, r, ldx, GRAM_BOX_COLS, GRAM_BOX_ROWS);
    if (e == cudaSuccess) e = encode_rows(&t.m[TMAP_GQ], any, K, r, ldq, GRAM_BOX_COLS, GRAM_BOX_ROWS);
    if (e != cudaSuccess) return e;
    k_tmaps<<<(B + 127) / 128, 128, 0, st>>>(p, B, t, maps);
    return cudaGetLastError();
}

}  // namespace spq
