// The Gram's fixed-order reduction over splits.
//
// k_gram_reduce: G = the sum of the split partials of k_gram_tc (128 x 128 tiles of the upper triangle) in split
// order, kept in float-float (about 44 bits, where tri.py:375 sums its splits in fp64: P.sum(0, float64).float()),
// rounded to fp32 once and mirrored; with make_D it
// writes D = 0.5 (I - G) instead (kcholqr.py:21).  Without make_D it also writes, per strip, the fp64 sum of the
// squares of the G entries it wrote (every entry of G is written exactly once): the Cholesky adds these partial sums
// in a fixed order for ||G||_F (kcholqr.py:107).
#include "kernels.h"

namespace spq {

// One CTA = a strip of 32 rows of one upper tile: the split sums of the strip go to shared memory (LT threads, one
// float4 of the strip per thread and step: 1024 threads when the grid is small, so that all of a thread's split loads
// are in flight together, 256 otherwise), then the first 256 threads write G row by row (coalesced) and, transposed,
// column by column (also coalesced), summing the squares of what they write in a fixed order.  The results do not
// depend on LT.  In a diagonal tile the tensor cores give (a, c)
// and (c, a) from the same products in different roles, which need not round alike: the upper element alone defines
// both, so G is exactly symmetric.
constexpr int RSTRIP = 32;

constexpr int WTHREADS = 256;   // writers of G (their order defines the strip's sum of squares)

template <int LT>
__global__ void __launch_bounds__(LT) k_gram_reduce(const float* __restrict__ P, int n, GramPlan gp, int make_D,
                                                     float* __restrict__ G, double* __restrict__ sq) {
    constexpr int T = GRAM_TILE;
    const int tile = blockIdx.x / (T / RSTRIP), r0 = (blockIdx.x % (T / RSTRIP)) * RSTRIP, b = blockIdx.y;
    int ti, tj;
    upper_tile(tile, gp.nt, ti, tj);
    const bool diag = ti == tj;
    __shared__ float S[RSTRIP][T + 1];
    const float* src = P + (size_t)b * gp.S * gp.tiles * (T * T) + (size_t)tile * (T * T) + (size_t)r0 * T;
    const size_t split_stride = (size_t)gp.tiles * (T * T);
    // 32 x 128 sums, a float4 of one row per thread and step
    for (int q = threadIdx.x; q < RSTRIP * T / 4; q += LT) {
        const int r = q / (T / 4), c = 4 * (q % (T / 4));
        // float-float sums (B200 converts fp32 to fp64 slowly), eight splits' loads in flight at a time, split order
        float h[4] = {0.f, 0.f, 0.f, 0.f}, l[4] = {0.f, 0.f, 0.f, 0.f};
        for (int sp0 = 0; sp0 < gp.S; sp0 += 8) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (sp0 + u < gp.S)
                    v[u] = __ldcg(reinterpret_cast<const float4*>(src + (size_t)(sp0 + u) * split_stride + (size_t)r * T + c));
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (sp0 + u < gp.S) {
                    ff_add(h[0], l[0], v[u].x);
                    ff_add(h[1], l[1], v[u].y);
                    ff_add(h[2], l[2], v[u].z);
                    ff_add(h[3], l[3], v[u].w);
                }
        }
        const double t0 = ff_value(h[0], l[0]), t1 = ff_value(h[1], l[1]), t2 = ff_value(h[2], l[2]),
                     t3 = ff_value(h[3], l[3]);
        const int a = ti * T + r0 + r;
        float g[4] = {__double2float_rn(t0), __double2float_rn(t1), __double2float_rn(t2), __double2float_rn(t3)};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (make_D) g[i] = __fmul_rn(__fsub_rn(a == tj * T + c + i ? 1.0f : 0.0f, g[i]), 0.5f);
            S[r][c + i] = g[i];
        }
    }
    __syncthreads();
    if (threadIdx.x >= WTHREADS) return;
    double q = 0.0;   // squares of the entries this thread writes
    // rows: G[a][c]; in a diagonal tile only c >= a
    for (int e = threadIdx.x; e < RSTRIP * T; e += WTHREADS) {
        const int r = e / T, c = e % T;
        const int a = ti * T + r0 + r, cg = tj * T + c;
        if (a >= n || cg >= n || (diag && cg < a)) continue;
        const float g = S[r][c];
        G[(size_t)b * n * n + (size_t)a * n + cg] = g;
        q = __fma_rn((double)g, (double)g, q);
    }
    // columns: G[c][a]; in a diagonal tile only c > a
    for (int e = threadIdx.x; e < RSTRIP * T; e += WTHREADS) {
        const int c = e / RSTRIP, r = e % RSTRIP;
        const int a = ti * T + r0 + r, cg = tj * T + c;
        if (a >= n || cg >= n || (diag && cg <= a)) continue;
        const float g = S[r][c];
        G[(size_t)b * n * n + (size_t)cg * n + a] = g;
        q = __fma_rn((double)g, (double)g, q);
    }
    if (sq) {   // fixed-order block sum: butterfly within each warp, then the warps in order
        __shared__ double wsum[WTHREADS / 32];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) q = __dadd_rn(q, __shfl_xor_sync(0xffffffffu, q, o));
        if ((threadIdx.x & 31) == 0) wsum[threadIdx.x >> 5] = q;
        asm volatile("bar.sync 1, %0;" ::"n"(WTHREADS));   // the writers only
        if (threadIdx.x == 0) {
            double t = wsum[0];
            for (int w = 1; w < WTHREADS / 32; ++w) t = __dadd_rn(t, wsum[w]);
            sq[(size_t)b * n + blockIdx.x] = t;
        }
    }
}

int gram_sq_parts(const GramPlan& gp) { return gp.tiles * (GRAM_TILE / RSTRIP); }

cudaError_t launch_gram_reduce(const float* P, int n, int B, const GramPlan& gp, int make_D, float* G, double* sq,
                               cudaStream_t st) {
    if ((long long)gram_sq_parts(gp) * B < 148)   // a small grid: every float4 of the strip its own thread
        k_gram_reduce<RSTRIP * GRAM_TILE / 4><<<dim3(gram_sq_parts(gp), B), RSTRIP * GRAM_TILE / 4, 0, st>>>(
            P, n, gp, make_D, G, make_D ? nullptr : sq);
    else
        k_gram_reduce<WTHREADS><<<dim3(gram_sq_parts(gp), B), WTHREADS, 0, st>>>(P, n, gp, make_D, G, make_D ? nullptr : sq);
    return cudaGetLastError();
}

}  // namespace spq
