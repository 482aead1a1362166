// Operand image of the tensor-core triangular solve: W_jk = -Li_j L_jk (k < j) and W_jj = Li_j, 32 x 32 tiles of the
// block lower triangle, split into tf32 hi + lo and laid out exactly as the solve's shared-memory operand tiles
// (K-major, 128B swizzle; 4 KB per part), so the solve copies them in without converting.  Tiles are grouped by block
// column k (wcol_off): the diagonal tile, then the hi parts of the tiles below it, then their lo parts, so that the
// tiles one finished block updates arrive in one copy and stack into one N = 32 (nb - 1 - k) operand.
//
// The solve's block recurrence  Y_j = (A_j - sum_{k<j} Y_k L_jk^T) Li_j^T  (candidates/tri.py:391-401) is evaluated as
// Y_j = A_j W_jj^T + sum_{k<j} Y_k W_jk^T: the same operation, with the diagonal-tile inverse applied to the
// coefficients first; each W_jk is one fp64-accumulated 32 x 32 product, rounded once to fp32.
#include "kernels.h"
#include "tc.cuh"

namespace spq {

__global__ void __launch_bounds__(256) k_trsm_w(const float* __restrict__ L_all, const float* __restrict__ Li_all, int n,
                                                char* __restrict__ W_all) {
    const int t = blockIdx.x, b = blockIdx.y;
    const int nb = n / TB;
    int j = 0;
    while ((j + 1) * (j + 2) / 2 <= t) ++j;
    const int k = t - j * (j + 1) / 2;
    const float* L = L_all + (size_t)b * n * n;
    const float* Li = Li_all + (size_t)b * n * TB;
    char* col = W_all + (size_t)b * wcol_off(nb, nb) + wcol_off(nb, k);
    char* hi = col;
    char* lo = col + 4096;
    if (k < j) {
        hi = col + 2 * 4096 + (size_t)(j - k - 1) * 4096;
        lo = hi + (size_t)(nb - 1 - k) * 4096;
    }
    // the tiles in fp64, converted once (B200 converts fp32 to fp64 at a tenth of its fp64 fma rate)
    __shared__ double sLi[TB][TB + 1], sL[TB][TB + 1];
    for (int e = threadIdx.x; e < TB * TB; e += blockDim.x) {
        const int r = e / TB, c = e % TB;
        sLi[r][c] = (double)Li[(size_t)(j * TB + r) * TB + c];
        sL[r][c] = (k < j) ? (double)L[(size_t)(j * TB + r) * n + k * TB + c] : 0.0;
    }
    __syncthreads();
    // thread: row r, columns 4 q .. 4 q + 3 (q = 0..7)
    const int r = threadIdx.x >> 3, q = threadIdx.x & 7;
    float w[4];
    if (k == j) {
#pragma unroll
        for (int i = 0; i < 4; ++i) w[i] = (float)sLi[r][4 * q + i];
    } else {
        // four chains, each over m in order; sLi[r][m] is loaded once for all four
        double acc[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll 8
        for (int m = 0; m < TB; ++m) {
            const double a = sLi[r][m];
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[i] = __fma_rn(a, sL[m][4 * q + i], acc[i]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) w[i] = -__double2float_rn(acc[i]);
    }
    tc::store2_at(hi, lo, tc::swz_off(r, q), make_float4(w[0], w[1], w[2], w[3]));
}

cudaError_t launch_trsm_w(const float* L, const float* Li, int n, int B, char* W, cudaStream_t st) {
    const int nb = n / TB;
    k_trsm_w<<<dim3(nb * (nb + 1) / 2, B), 256, 0, st>>>(L, Li, n, W);
    return cudaGetLastError();
}

}  // namespace spq
