// Split-K compensated Gram G = A^T A (A = s Y), its fixed-order reduction, and the row sums of squares of G.
//
// Follows candidates/tri.py:255-297 (gram_split) and :324-375 (gram_f): 64 x 64 output tiles of the upper triangle,
// the rows split into S ranges (the reference's split formula at 148 SMs, so every B200 gives the same bits), a
// 32-row fp32 FMA-chain dot per chunk, Kahan-compensated across the chunks of a split, an fp64 sum across splits
// in split order, rounded to fp32 and mirrored.  Columns beyond n are masked (the reference leaves them unmasked).
#include "kernels.h"

namespace spq {

GramPlan gram_plan(int K, int n) {
    GramPlan g;
    g.nt = (n + GT - 1) / GT;
    g.tiles = g.nt * (g.nt + 1) / 2;
    const int tp = 3 * NSM_SPLIT;
    int S = (tp + g.tiles - 1) / g.tiles;
    const int cap = (K + 4 * GK - 1) / (4 * GK);
    if (cap < S) S = cap;
    if (S < 1) S = 1;
    const int per = (K + S - 1) / S;
    g.KS = ((per + GK - 1) / GK) * GK;
    g.S = (K + g.KS - 1) / g.KS;
    return g;
}

__global__ void __launch_bounds__(256) k_gram_partial(PtrArg p, Src src, int K, int n, long long ld, GramPlan gp,
                                                      ScaleArg sc, float* __restrict__ P) {
    const int tile = blockIdx.x, sp = blockIdx.y, b = blockIdx.z;
    int ti, tj;
    upper_tile(tile, gp.nt, ti, tj);
    const MatPtr mp = p.tab ? p.tab[b] : p.one;
    const float* __restrict__ Y = (src == SRC_X) ? mp.X : mp.Q;
    float s = 1.0f;
    bool scaled = false;
    if (sc.maxbits) {
        s = pow2_scale(__uint_as_float(sc.maxbits[b]));
        scaled = true;
    } else if (sc.s) {
        s = sc.s[b];
        scaled = true;
    }
    const int k0 = sp * gp.KS;
    const int k1 = min(k0 + gp.KS, K);
    __shared__ __align__(16) float As[GK][GT];
    __shared__ __align__(16) float Bs[GK][GT];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int ca = ti * GT, cb = tj * GT;
    float acc[4][4], comp[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = comp[i][j] = 0.0f;

    for (int c0 = k0; c0 < k1; c0 += GK) {
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int e = threadIdx.x + q * 256;  // float4 index in the 32 x 64 chunk
            const int rr = e >> 4, cc = (e & 15) * 4;
            const int row = c0 + rr;
            float4 va = make_float4(0.f, 0.f, 0.f, 0.f), vb = va;
            if (row < k1) {
                if (ca + cc < n) va = __ldg(reinterpret_cast<const float4*>(Y + (long long)row * ld + ca + cc));
                if (cb + cc < n) vb = __ldg(reinterpret_cast<const float4*>(Y + (long long)row * ld + cb + cc));
            }
            if (scaled) {
                va.x = __fmul_rn(va.x, s); va.y = __fmul_rn(va.y, s); va.z = __fmul_rn(va.z, s); va.w = __fmul_rn(va.w, s);
                vb.x = __fmul_rn(vb.x, s); vb.y = __fmul_rn(vb.y, s); vb.z = __fmul_rn(vb.z, s); vb.w = __fmul_rn(vb.w, s);
            }
            *reinterpret_cast<float4*>(&As[rr][cc]) = va;
            *reinterpret_cast<float4*>(&Bs[rr][cc]) = vb;
        }
        __syncthreads();
        float part[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) part[i][j] = 0.0f;
#pragma unroll 8
        for (int k = 0; k < GK; ++k) {
            const float4 a4 = *reinterpret_cast<const float4*>(&As[k][ty * 4]);
            const float4 b4 = *reinterpret_cast<const float4*>(&Bs[k][tx * 4]);
            const float av[4] = {a4.x, a4.y, a4.z, a4.w};
            const float bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) part[i][j] = __fmaf_rn(av[i], bv[j], part[i][j]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float yv = __fsub_rn(part[i][j], comp[i][j]);
                const float t = __fadd_rn(acc[i][j], yv);
                comp[i][j] = __fsub_rn(__fsub_rn(t, acc[i][j]), yv);
                acc[i][j] = t;
            }
        __syncthreads();
    }
    float* out = P + ((size_t)(b * gp.S + sp) * gp.tiles + tile) * (GT * GT);
#pragma unroll
    for (int i = 0; i < 4; ++i)
        *reinterpret_cast<float4*>(out + (ty * 4 + i) * GT + tx * 4) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
}

__global__ void __launch_bounds__(256) k_gram_reduce(const float* __restrict__ P, int n, GramPlan gp, int make_D,
                                                     float* __restrict__ G) {
    const int tile = blockIdx.x, b = blockIdx.y;
    int ti, tj;
    upper_tile(tile, gp.nt, ti, tj);
    float* Gb = G + (size_t)b * n * n;
    for (int e = threadIdx.x; e < GT * GT; e += blockDim.x) {
        const int a = ti * GT + (e >> 6), c = tj * GT + (e & 63);
        if (a >= n || c >= n) continue;
        double t = 0.0;
        const float* src = P + (size_t)b * gp.S * gp.tiles * (GT * GT) + (size_t)tile * (GT * GT) + e;
        for (int sp = 0; sp < gp.S; ++sp) t = __dadd_rn(t, (double)src[(size_t)sp * gp.tiles * (GT * GT)]);
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

cudaError_t launch_gram_partial(PtrArg p, Src src, int K, int n, long long ld, int B, const GramPlan& gp, ScaleArg sc,
                                float* P, cudaStream_t st) {
    k_gram_partial<<<dim3(gp.tiles, gp.S, B), 256, 0, st>>>(p, src, K, n, ld, gp, sc, P);
    return cudaGetLastError();
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
