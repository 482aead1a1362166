// Row-block kernel for n > 256: the blocked triangular solve Y = (s X + eps Z) L^-T.
//
// Each CTA owns BM = 64 rows and keeps them (all n columns) in shared memory for the whole kernel, so it runs in
// place on Q: rows are read once, finished in shared memory, and written once; no other CTA touches them.
//
// trsm follows candidates/tri.py:378-403 (_trsm_f_kernel): 32-column blocks j in order; acc = s x (+ eps z); for each
// earlier block k, acc -= (Y_k L[j, k]^T) with that dot as one FMA chain; then Y_j = acc Li_j^T.
// Thread map: 256 threads = 32 row pairs x 8 column groups of 4; shared rows padded to n + 1 floats (no bank
// conflicts for the column-group reads).
#include "kernels.h"

namespace spq {

constexpr int BM = 64;

__device__ __forceinline__ float load_scale(ScaleArg sc, int b, bool& scaled) {
    if (sc.maxbits) {
        scaled = true;
        return pow2_scale(__uint_as_float(sc.maxbits[b]));
    }
    if (sc.s) {
        scaled = true;
        return sc.s[b];
    }
    scaled = false;
    return 1.0f;
}

// Ys[rr][c] = s * x (+ eps * z) for the CTA's rows (rows past K are zero)
__device__ __forceinline__ void load_rows(float* Ys, int ldy, const float* Xin, long long ldin, int row0, int K, int n,
                                          bool scaled, float s, const float* Z, float eps) {
    const int n4 = n / 4;
    for (int e = threadIdx.x; e < BM * n4; e += blockDim.x) {
        const int rr = e / n4, c = (e - rr * n4) * 4;
        const int row = row0 + rr;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (row < K) {
            v = *reinterpret_cast<const float4*>(Xin + (long long)row * ldin + c);
            if (scaled) {
                v.x = __fmul_rn(v.x, s); v.y = __fmul_rn(v.y, s); v.z = __fmul_rn(v.z, s); v.w = __fmul_rn(v.w, s);
            }
            if (Z) {
                const float4 z = __ldg(reinterpret_cast<const float4*>(Z + (long long)row * n + c));
                v.x = __fadd_rn(v.x, __fmul_rn(eps, z.x));
                v.y = __fadd_rn(v.y, __fmul_rn(eps, z.y));
                v.z = __fadd_rn(v.z, __fmul_rn(eps, z.z));
                v.w = __fadd_rn(v.w, __fmul_rn(eps, z.w));
            }
        }
        float* d = Ys + rr * ldy + c;
        d[0] = v.x; d[1] = v.y; d[2] = v.z; d[3] = v.w;
    }
}

__device__ __forceinline__ void store_rows(const float* Ys, int ldy, float* Qout, long long ldq, int row0, int K, int n) {
    const int n4 = n / 4;
    for (int e = threadIdx.x; e < BM * n4; e += blockDim.x) {
        const int rr = e / n4, c = (e - rr * n4) * 4;
        const int row = row0 + rr;
        if (row >= K) continue;
        const float* s = Ys + rr * ldy + c;
        *reinterpret_cast<float4*>(Qout + (long long)row * ldq + c) = make_float4(s[0], s[1], s[2], s[3]);
    }
}

__global__ void __launch_bounds__(256) k_trsm(PtrArg p, Src src, int K, int n, long long ldx, long long ldq,
                                              const float* __restrict__ Z, ScaleArg sc, float eps,
                                              const float* __restrict__ L_all, const float* __restrict__ Li_all) {
    extern __shared__ __align__(16) float sm[];
    const int ldy = n + 1;
    float* Ys = sm;                 // [BM][n + 1]
    float* Lp = Ys + BM * ldy;      // [32][n + 1]: rows j..j+31 of L, columns 0..j-1
    float* Lis = Lp + TB * ldy;     // [32][33]:   Li_j
    const int b = blockIdx.y;
    const MatPtr mp = p.tab ? p.tab[b] : p.one;
    const float* Xin = (src == SRC_X) ? mp.X : mp.Q;
    const long long ldin = (src == SRC_X) ? ldx : ldq;
    const float* L = L_all + (size_t)b * n * n;
    const float* Li = Li_all + (size_t)b * n * TB;
    bool scaled;
    const float s = load_scale(sc, b, scaled);
    const int row0 = blockIdx.x * BM;
    load_rows(Ys, ldy, Xin, ldin, row0, K, n, scaled, s, Z, eps);

    const int rp = threadIdx.x >> 3, cg = threadIdx.x & 7;
    const float* y0 = Ys + (2 * rp) * ldy;
    const float* y1 = y0 + ldy;
    for (int j = 0; j < n; j += TB) {
        for (int e = threadIdx.x; e < TB * j; e += blockDim.x) {
            const int c = e / j, m = e - c * j;
            Lp[c * ldy + m] = __ldg(L + (size_t)(j + c) * n + m);
        }
        for (int e = threadIdx.x; e < TB * TB; e += blockDim.x) Lis[(e >> 5) * (TB + 1) + (e & 31)] = __ldg(Li + (size_t)j * TB + e);
        __syncthreads();
        float acc[2][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            acc[0][i] = y0[j + cg * 4 + i];
            acc[1][i] = y1[j + cg * 4 + i];
        }
        for (int k = 0; k < j; k += TB) {
            float d[2][4];
#pragma unroll
            for (int i = 0; i < 4; ++i) d[0][i] = d[1][i] = 0.0f;
#pragma unroll 8
            for (int m = 0; m < TB; ++m) {
                const float a0 = y0[k + m], a1 = y1[k + m];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float l = Lp[(cg * 4 + i) * ldy + k + m];
                    d[0][i] = __fmaf_rn(a0, l, d[0][i]);
                    d[1][i] = __fmaf_rn(a1, l, d[1][i]);
                }
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                acc[0][i] = __fsub_rn(acc[0][i], d[0][i]);
                acc[1][i] = __fsub_rn(acc[1][i], d[1][i]);
            }
        }
        float* w0 = Ys + (2 * rp) * ldy;
        float* w1 = w0 + ldy;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            w0[j + cg * 4 + i] = acc[0][i];
            w1[j + cg * 4 + i] = acc[1][i];
        }
        __syncthreads();
        float out[2][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) out[0][i] = out[1][i] = 0.0f;
#pragma unroll 8
        for (int c = 0; c < TB; ++c) {
            const float a0 = y0[j + c], a1 = y1[j + c];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float li = Lis[(cg * 4 + i) * (TB + 1) + c];
                out[0][i] = __fmaf_rn(a0, li, out[0][i]);
                out[1][i] = __fmaf_rn(a1, li, out[1][i]);
            }
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            w0[j + cg * 4 + i] = out[0][i];
            w1[j + cg * 4 + i] = out[1][i];
        }
    }
    __syncthreads();
    store_rows(Ys, ldy, mp.Q, ldq, row0, K, n);
}

static size_t trsm_smem(int n) { return sizeof(float) * ((size_t)(BM + TB) * (n + 1) + TB * (TB + 1)); }

cudaError_t launch_trsm(PtrArg p, Src src, int K, int n, long long ldx, long long ldq, int B, const float* Z,
                        ScaleArg sc, float eps, const float* L, const float* Li, cudaStream_t st) {
    const size_t smem = trsm_smem(n);
    cudaError_t e = cudaFuncSetAttribute(k_trsm, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    k_trsm<<<dim3(cdiv(K, BM), B), 256, smem, st>>>(p, src, K, n, ldx, ldq, Z, sc, eps, L, Li);
    return cudaGetLastError();
}

}  // namespace spq
