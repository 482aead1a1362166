// Newton-Schulz update Y <- Y + Y D (candidates/kcholqr.py:22, torch.addmm(Y, Y, D)) on the tcgen05 tensor cores.
//
// One CTA = 128 rows of one matrix and all N = n output columns (n <= 256; wider matrices use k_ns_update, which
// holds whole rows in shared memory).  The contraction runs over the n columns of Y in chunks of 32: per chunk the 256
// threads load the row block Y[rows, k0 .. k0+32) and the panel D[cols, k0 .. k0+32) (D is symmetric, so row c of D is
// column c), split every value into tf32 hi + lo and store both K-major into 128B-swizzled shared tiles (Y's rows and
// D's rows are already K-contiguous); one thread issues per k-step of 8 the products hi.hi, hi.lo and lo.hi
// (tcgen05.mma M128 N<=256 K8).  The epilogue adds, per element, y + acc in fp32 and writes the row block back in
// place (the CTA owns its rows; every other CTA reads only D).
// Two CTAs share an SM (one operand buffer of at most 96 KB and at most 256 TMEM columns each), so one CTA's loads and
// barriers overlap the other's products.  For n <= 128 hi.hi and the two cross terms go to separate accumulators; for
// wider n all three share one.
// Accuracy: |Y D| is at most about 1e-2 |Y| (||D||_2 <= 1e-2 across the reference's cases), so the 3xTF32 products
// and the tensor core's fp32 accumulation (truncating, at most one ulp of the accumulator per k-step) leave errors
// below one ulp of Y in the first polish step and far below it in the second, where ||D||_2 is about 1e-4.
#include "kernels.h"
#include "tc.cuh"

namespace spq {

namespace {
constexpr int NT = 256;
constexpr int ROWS = 128;       // M
constexpr int CHUNK = 32;       // K per chunk (4 MMA k-steps)
constexpr int A_TILE = ROWS * 128;   // 128 rows x 32 tf32 (K-major, 128B swizzle)
constexpr int ERR_TIMEOUT = 0x20;

template <int N> constexpr int b_tile() { return N * 128; }
template <int N> constexpr int buf_bytes() { return 2 * A_TILE + 2 * b_tile<N>(); }   // A hi, lo; B hi, lo
template <int N> constexpr int smem_bytes() { return buf_bytes<N>() + 1024 + 1024; }
template <int N> constexpr bool split_acc() { return 2 * N <= 256; }
}  // namespace

// N: output columns per pass (<= 256, a multiple of 32)
template <int N>
__global__ void __launch_bounds__(NT, 2) k_ns_tc(PtrArg p, int K, int n, long long ldq, const float* __restrict__ D_all,
                                                 int* __restrict__ status) {
    constexpr int BUF = buf_bytes<N>();
    constexpr int BT = b_tile<N>();
    constexpr bool SPLIT = split_acc<N>();
    constexpr uint32_t TCOLS = (SPLIT ? 2 * N : N) <= 32 ? 32 : (SPLIT ? 2 * N : N) <= 64 ? 64 : (SPLIT ? 2 * N : N) <= 128 ? 128 : 256;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    char* const buf0 = reinterpret_cast<char*>(sm);   // one operand buffer: A hi, A lo, B hi, B lo
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + BUF);   // [0] operand buffer free
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + BUF + 64);

    const int b = blockIdx.y;
    const int row0 = blockIdx.x * ROWS;
    const MatPtr mp = p.tab ? p.tab[b] : p.one;
    float* Q = mp.Q;
    const float* D = D_all + (size_t)b * n * n;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nchunks = n / CHUNK;

    if (warp == 0) tc::tmem_alloc(tmem_slot, TCOLS);
    if (threadIdx.x == 0) {
        tc::mbar_init(&bars[0], 1);
        tc::mbar_fence_init();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint32_t idesc = tc::idesc_tf32(ROWS, N);

    // K-major stores: a warp writes 8 consecutive rows x 4 k-quads (one half of a 1024-byte swizzle atom)
    const int qq = (warp >> 2) * 4 + (lane >> 3);    // k-quad 0..7 (4 floats each)
    const int rr = lane & 7;
    bool ok = true;

    constexpr int NB = N / 32;
    float4 ra[4], rb[NB];   // one chunk: A: 4 row slots, B: N / 32 row slots (this thread's k-quad qq)
    auto load = [&](int c) {
        const int k = c * CHUNK + 4 * qq;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int row = row0 + 8 * ((warp & 3) * 4 + j) + rr;
            ra[j] = (row < K) ? *reinterpret_cast<const float4*>(Q + (long long)row * ldq + k) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int j = 0; j < NB; ++j) {
            const int col = 8 * ((warp & 3) * NB + j) + rr;
            rb[j] = __ldg(reinterpret_cast<const float4*>(D + (size_t)col * n + k));
        }
    };
    load(0);
    for (int c = 0; c < nchunks; ++c) {
        if (c >= 1) ok = tc::mbar_wait(&bars[0], (uint32_t)((c - 1) & 1));   // the previous chunk's products are done
        ok = __syncthreads_and(ok);
        if (!ok) break;
#pragma unroll
        for (int j = 0; j < 4; ++j) tc::store2_at(buf0, buf0 + A_TILE, tc::swz_off(8 * ((warp & 3) * 4 + j) + rr, qq), ra[j]);
#pragma unroll
        for (int j = 0; j < NB; ++j)
            tc::store2_at(buf0 + 2 * A_TILE, buf0 + 2 * A_TILE + BT, tc::swz_off(8 * ((warp & 3) * NB + j) + rr, qq), rb[j]);
        tc::fence_async_smem();
        if (c + 1 < nchunks) load(c + 1);
        __syncthreads();
        if (threadIdx.x == 0) {
            tc::fence_after_sync();
            const uint32_t abase = tc::smem_u32(buf0), bbase = abase + 2 * A_TILE;
            const uint32_t dbig = tmem, dsmall = SPLIT ? tmem + N : tmem;
#pragma unroll 1
            for (int k = 0; k < CHUNK / 8; ++k) {
                const uint32_t acc_in = (c > 0 || k > 0) ? 1u : 0u;
                const uint64_t ahi = tc::sdesc_k128(abase + 32 * k), alo = tc::sdesc_k128(abase + A_TILE + 32 * k);
                const uint64_t bhi = tc::sdesc_k128(bbase + 32 * k), blo = tc::sdesc_k128(bbase + BT + 32 * k);
                tc::mma_tf32(dbig, ahi, bhi, idesc, acc_in);
                tc::mma_tf32(dsmall, ahi, blo, idesc, SPLIT ? acc_in : 1u);
                tc::mma_tf32(dsmall, alo, bhi, idesc, 1u);
            }
            tc::mma_commit(&bars[0]);
        }
    }
    if (ok) ok = __syncthreads_and(tc::mbar_wait(&bars[0], (uint32_t)((nchunks - 1) & 1)));
    if (ok) {
        // epilogue: out = y + acc for this thread's row and 32-column slices
        tc::fence_after_sync();
        const int m = (warp & 3) * 32 + lane;
        const int row = row0 + m;
        const uint32_t lanebase = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        for (int sl = (warp >> 2); sl < N / 32; sl += 2) {
            float big[32], small[32];
            tc::tmem_ld32(lanebase + 32 * sl, big);
            if constexpr (SPLIT) tc::tmem_ld32(lanebase + N + 32 * sl, small);
            tc::tmem_wait_ld();
            if (row < K) {
                float* qr = Q + (long long)row * ldq + 32 * sl;
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                    const float4 y = *reinterpret_cast<const float4*>(qr + i);
                    float a0 = big[i], a1 = big[i + 1], a2 = big[i + 2], a3 = big[i + 3];
                    if constexpr (SPLIT) {
                        a0 = __fadd_rn(a0, small[i]);
                        a1 = __fadd_rn(a1, small[i + 1]);
                        a2 = __fadd_rn(a2, small[i + 2]);
                        a3 = __fadd_rn(a3, small[i + 3]);
                    }
                    *reinterpret_cast<float4*>(qr + i) =
                        make_float4(__fadd_rn(y.x, a0), __fadd_rn(y.y, a1), __fadd_rn(y.z, a2), __fadd_rn(y.w, a3));
                }
            }
        }
    } else if (threadIdx.x == 0) {
        tc::mbar_wait(&bars[0], (uint32_t)((nchunks - 1) & 1));   // let issued products finish before TMEM is freed
    }
    if (!ok && threadIdx.x == 0) atomicOr(status, ERR_TIMEOUT);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 0) tc::tmem_dealloc(tmem, TCOLS);
}

template <int N>
static cudaError_t launch_n(PtrArg p, int K, int n, long long ldq, int B, const float* D, int* status, cudaStream_t st) {
    constexpr int smem = smem_bytes<N>();
    cudaError_t e = cudaFuncSetAttribute(k_ns_tc<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    k_ns_tc<N><<<dim3((K + ROWS - 1) / ROWS, B), NT, smem, st>>>(p, K, n, ldq, D, status);
    return cudaGetLastError();
}

cudaError_t launch_ns_tc(PtrArg p, int K, int n, long long ldq, int B, const float* D, int* status, cudaStream_t st) {
    switch (n) {
        case 32: return launch_n<32>(p, K, n, ldq, B, D, status, st);
        case 64: return launch_n<64>(p, K, n, ldq, B, D, status, st);
        case 96: return launch_n<96>(p, K, n, ldq, B, D, status, st);
        case 128: return launch_n<128>(p, K, n, ldq, B, D, status, st);
        case 160: return launch_n<160>(p, K, n, ldq, B, D, status, st);
        case 192: return launch_n<192>(p, K, n, ldq, B, D, status, st);
        case 224: return launch_n<224>(p, K, n, ldq, B, D, status, st);
        case 256: return launch_n<256>(p, K, n, ldq, B, D, status, st);
        default: return cudaErrorInvalidValue;   // n > 256 runs k_ns_update
    }
}

}  // namespace spq
