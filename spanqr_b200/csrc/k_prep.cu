// Call set-up (pointer tables, zeroed accumulators) and max |X| per matrix.
#include <atomic>

#include "kernels.h"

namespace spq {

namespace {
std::atomic<int> g_nsm[64];
}

cudaError_t sm_count(int* nsm) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaDeviceGetAttribute(nsm, cudaDevAttrMultiProcessorCount, dev);
    int v = g_nsm[dev].load(std::memory_order_relaxed);
    if (v == 0) {
        e = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        g_nsm[dev].store(v, std::memory_order_relaxed);
    }
    *nsm = v;
    return cudaSuccess;
}

__global__ void k_setup_strided(MatPtr* tab, const float* X, long long sX, float* Q, long long sQ, int B,
                                uint32_t* maxbits, int* status) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B) {
        tab[b].X = X + (long long)b * sX;
        tab[b].Q = Q + (long long)b * sQ;
        maxbits[b] = 0u;
    }
    if (b == 0 && status) status[0] = 0;   // null: keep the status of the calls before (block Gram-Schmidt)
}

__global__ void k_setup_array(MatPtr* tab, const float* const* dX, float* const* dQ, int B, uint32_t* maxbits,
                              int* status) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B) {
        tab[b].X = dX[b];
        tab[b].Q = dQ[b];
        maxbits[b] = 0u;
    }
    if (b == 0) status[0] = 0;
}

constexpr int HOST_CHUNK = 128;   // pointer pairs per set-up launch (2 KB of kernel parameters)

struct PtrChunk {
    MatPtr m[HOST_CHUNK];
};

__global__ void k_setup_chunk(MatPtr* tab, PtrChunk c, int b0, int nb, uint32_t* maxbits, int* status) {
    const int i = threadIdx.x;
    if (i < nb) {
        tab[b0 + i] = c.m[i];
        maxbits[b0 + i] = 0u;
    }
    if (b0 == 0 && i == 0) status[0] = 0;
}

// max |x| over X[b] (K x r, leading dimension ldx) as bits; NaN wins (kcholqr.py:102 vector_norm(ord=inf)).
// The maximum is order-independent, so the atomic combine is deterministic.
__global__ void __launch_bounds__(256) k_absmax(PtrArg p, int K, int r, long long ldx, uint32_t* maxbits) {
    const int b = blockIdx.y;
    const float* X = p.tab ? p.tab[b].X : p.one.X;
    const long long n4 = (long long)K * r / 4;
    const int r4 = r / 4;
    uint32_t m = 0u;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
        const long long row = i / r4;
        const int col = (int)(i - row * r4) * 4;
        const float4 v = __ldg(reinterpret_cast<const float4*>(X + row * ldx + col));
        m = max(m, max(max(abs_bits(v.x), abs_bits(v.y)), max(abs_bits(v.z), abs_bits(v.w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    __shared__ uint32_t red[8];
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t t = red[0];
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) t = max(t, red[w]);
        atomicMax(maxbits + b, t);
    }
}

int setup_host_launches(int B) { return (B + HOST_CHUNK - 1) / HOST_CHUNK; }

const void* setup_strided_kernel() { return reinterpret_cast<const void*>(&k_setup_strided); }

cudaError_t launch_setup_strided(MatPtr* tab, const float* X, long long sX, float* Q, long long sQ, int B,
                                 uint32_t* maxbits, int* status, cudaStream_t st) {
    k_setup_strided<<<cdiv(B, 128), 128, 0, st>>>(tab, X, sX, Q, sQ, B, maxbits, status);
    return cudaGetLastError();
}

cudaError_t launch_setup_array(MatPtr* tab, const float* const* dX, float* const* dQ, int B, uint32_t* maxbits,
                               int* status, cudaStream_t st) {
    k_setup_array<<<cdiv(B, 128), 128, 0, st>>>(tab, dX, dQ, B, maxbits, status);
    return cudaGetLastError();
}

cudaError_t launch_setup_host(MatPtr* tab, const float* const* hX, float* const* hQ, int B, uint32_t* maxbits,
                              int* status, cudaStream_t st) {
    for (int b0 = 0; b0 < B; b0 += HOST_CHUNK) {
        PtrChunk c;
        const int nb = (B - b0 < HOST_CHUNK) ? B - b0 : HOST_CHUNK;
        for (int i = 0; i < HOST_CHUNK; ++i) c.m[i] = (i < nb) ? MatPtr{hX[b0 + i], hQ[b0 + i]} : MatPtr{nullptr, nullptr};
        k_setup_chunk<<<1, HOST_CHUNK, 0, st>>>(tab, c, b0, nb, maxbits, status);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t launch_absmax(PtrArg p, int K, int r, long long ldx, int B, uint32_t* maxbits, cudaStream_t st) {
    const long long n4 = (long long)K * r / 4;
    int blocks = (int)((n4 + 256 * 8 - 1) / (256 * 8));   // ~8 float4 per thread
    if (blocks < 1) blocks = 1;
    if (blocks > 1024) blocks = 1024;
    k_absmax<<<dim3(blocks, B), 256, 0, st>>>(p, K, r, ldx, maxbits);
    return cudaGetLastError();
}

}  // namespace spq
