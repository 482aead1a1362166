// The Gram's fixed-order reduction over splits, and the row sums of squares of G.
//
// k_gram_reduce: G = fp64 sum of the split partials of k_gram_tc (128 x 128 tiles of the upper triangle) in split
// order, rounded to fp32 and mirrored, as tri.py:375 sums its splits (P.sum(0, float64).float()); with make_D it
// writes D = 0.5 (I - G) instead (kcholqr.py:21).
#include "kernels.h"

namespace spq {

__global__ void __launch_bounds__(256) k_gram_reduce(const float* __restrict__ P, int n, GramPlan gp, int make_D,
                                                     float* __restrict__ G) {
    const int tile = blockIdx.x, b = blockIdx.y;
    int ti, tj;
    upper_tile(tile, gp.nt, ti, tj);
    float* Gb = G + (size_t)b * n * n;
    constexpr int T = GRAM_TILE;
    for (int e = threadIdx.x; e < T * T; e += blockDim.x) {
        const int a = ti * T + e / T, c = tj * T + e % T;
        if (a >= n || c >= n) continue;
        // in a diagonal tile the tensor cores give (a, c) and (c, a) from the same products in different roles,
        // which need not round alike: the upper element alone defines both, so G is exactly symmetric
        if (ti == tj && a > c) continue;
        double t = 0.0;
        const float* src = P + (size_t)b * gp.S * gp.tiles * (T * T) + (size_t)tile * (T * T) + e;
        for (int sp = 0; sp < gp.S; ++sp) t = __dadd_rn(t, (double)src[(size_t)sp * gp.tiles * (T * T)]);
        float g = __double2float_rn(t);
        if (make_D) g = __fmul_rn(__fsub_rn(a == c ? 1.0f : 0.0f, g), 0.5f);
        Gb[(size_t)a * n + c] = g;
        Gb[(size_t)c * n + a] = g;
    }
}

// rowsq[b][a] = sum over c of G[b][a][c]^2 in fp64, c in order; G is exactly symmetric, so column a is read
// (coalesced) in place of row a.
__global__ void __launch_bounds__(128) k_rowsq(const float* __restrict__ G, int n, double* __restrict__ rowsq) {
    const int b = blockIdx.y;
    const int a = blockIdx.x * blockDim.x + threadIdx.x;
    if (a >= n) return;
    const float* Gb = G + (size_t)b * n * n;
    double row = 0.0;
    for (int c = 0; c < n; ++c) {
        const double g = (double)Gb[(size_t)c * n + a];
        row = __dadd_rn(row, __dmul_rn(g, g));
    }
    rowsq[(size_t)b * n + a] = row;
}

cudaError_t launch_gram_reduce(const float* P, int n, int B, const GramPlan& gp, int make_D, float* G,
                               cudaStream_t st) {
    k_gram_reduce<<<dim3(gp.tiles, B), 256, 0, st>>>(P, n, gp, make_D, G);
    return cudaGetLastError();
}

cudaError_t launch_rowsq(const float* G, int n, int B, double* rowsq, cudaStream_t st) {
    k_rowsq<<<dim3(cdiv(n, 128), B), 128, 0, st>>>(G, n, rowsq);
    return cudaGetLastError();
}

}  // namespace spq
