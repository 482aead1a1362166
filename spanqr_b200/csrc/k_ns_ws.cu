// Newton-Schulz update Q <- Q + Q D (candidates/kcholqr.py:22, torch.addmm(Y, Y, D)) for n <= 256 on the tcgen05
// tensor cores, 3xTF32 (hi.hi into one TMEM accumulator, hi.lo + lo.hi into a second).
//
// k_d_image splits D (symmetric, from k_gram_reduce) once per matrix into tf32 hi/lo operand tiles laid out as the
// update's shared-memory B operand: for each chunk of 32 contraction indices and each column half, the half's rows c
// (row c of D is column c) x 32 k, K-major with the 128-byte swizzle, hi part then lo part, so that k_ns_ws streams
// each chunk of each half with one bulk copy.
// One CTA = 128 rows of one matrix, all n output columns, in nh = 1 (n <= 256) or 2 column halves of N = n / nh
// (TMEM holds the large and small accumulators of at most 256 columns); warp roles: 0-3 epilogue (TMEM lanes = rows:
// y + acc), 4-7 convert (raw 32-column tile of Q by TMA -> tf32 hi | lo, K-major), 8 products (one thread, fixed
// order), 9 copies (one thread).  The last half is written in place; an earlier half still feeds the later halves'
// products, so its new values wait in `scratch` and are copied in after the last half.
// Product mode (MODE 1, for the triangular solve of n > 256): the same pipeline computes only the accumulator
// sum_{k < j0} Y_k [W_{j0, k}; ...; W_{j0+nbp-1, k}]^T from the solve's W image (A = the first 32 j0 columns of Q,
// B = the stacked W tiles of block column k) and writes it to `scratch` (K x 256 per matrix).
// Projection mode (MODE 2, block Gram-Schmidt for r > 512, candidates/kbig.py:66-95 W - P (P^T W)): A = the first j0
// columns of Q (the finished blocks P), B = -T (T = P^T W, k_band_image), N = 256; the result is added to the block
// W = Q[:, j0 .. j0 + 256) in place.  Accuracy: |Q D| is about 1e-2 |Q| or less, so 3xTF32 and the truncating fp32
// accumulation leave errors below one ulp of Q.
#include "kernels.h"
#include "tc.cuh"

namespace spq {

namespace {
constexpr int NT = 320;
constexpr int ROWS = 128;
constexpr int CH = 32;                          // contraction indices per chunk
constexpr int YT = ROWS * CH * 4;               // 128 x 32 fp32 / tf32: 16 KB
constexpr int DPART = 256 * CH * 4;             // up to 256 rows of D x 32 k: 32 KB
constexpr int OFF_RAW = 0;                      // two raw A tiles
constexpr int OFF_AOP = OFF_RAW + 2 * YT;       // two A operand stages [hi | lo]
constexpr int OFF_DB = OFF_AOP + 2 * 2 * YT;    // two D operand stages [hi | lo]
constexpr int OFF_BAR = OFF_DB + 2 * 2 * DPART;
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;
constexpr uint32_t TCOLS = 512;                 // large at 0, small at 256
constexpr int ERR_TIMEOUT = 0x20;
// mbarriers (x2 per stage): raw A landed, raw A read (128 arrivals), A operands written (128 arrivals), D chunk
// landed, chunk products done; then a half's products done, its accumulators read (128 arrivals), error drain.
// Every waiter steps through a barrier's phases in order from phase 0, and no barrier can run two phases ahead of a
// waiter.
enum { B_RAW = 0, B_RAWFREE = 2, B_OP = 4, B_D = 6, B_FREE = 8, B_DONE = 10, B_TFREE = 11, B_FIN = 12, NBAR = 13 };
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
static_assert(TMAP_BOX_COLS == CH && TMAP_BOX_ROWS == ROWS, "one TMA box is one 128-row tile of a chunk");
__device__ __forceinline__ uint32_t ring_parity(int c) { return (uint32_t)((c >> 1) & 1); }
}  // namespace

// one thread: row c of D, k-quad q of chunk kc
__global__ void k_d_image(const float* __restrict__ D_all, int n, char* __restrict__ img_all) {
    const int b = blockIdx.y;
    const int e = blockIdx.x * blockDim.x + threadIdx.x;   // (kc, c, q)
    const int nq = n / 4;
    if (e >= n * nq) return;
    const int c = e / nq, kq = e % nq, kc = kq / 8, q = kq % 8;
    const int N = n > 256 ? n / 2 : n, h = c / N, rr = c % N;   // column half and row within it
    const float4 v = *reinterpret_cast<const float4*>(D_all + (size_t)b * n * n + (size_t)c * n + 4 * kq);
    char* part = img_all + (size_t)b * ns_dimg_bytes(n) + (size_t)kc * 2 * n * 128 + (size_t)h * 2 * N * 128;
    tc::store2_at(part, part + (size_t)N * 128, tc::swz_off(rr, q), v);
}

template <int NH, int MODE>   // NH: column halves (1 for n <= 256, 2 above); MODE: 0 update, 1 solve panel product,
                              // 2 projection
__global__ void __launch_bounds__(NT, 1) k_ns_ws(PtrArg p, int K, int n, long long ldq, const char* __restrict__ maps,
                                                 const char* __restrict__ img_all, float* __restrict__ scratch,
                                                 int* __restrict__ status, int ncontr, int Nout, int j0) {
    extern __shared__ unsigned char smem_raw[];
    char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    char* const RAW = sm + OFF_RAW;
    char* const AOP = sm + OFF_AOP;
    char* const DB = sm + OFF_DB;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 128);
    volatile int* err = reinterpret_cast<volatile int*>(sm + OFF_BAR + 132);

    const int b = blockIdx.y;
    const int row0 = blockIdx.x * ROWS;
    const int nchunks = ncontr / CH;              // chunks of the contraction
    constexpr int nh = NH;
    const int N = Nout;                           // width of a column half (MODE 1: of the panel product)
    const int oc0 = MODE == 2 ? j0 : 0;           // the output's first column
    const int total = nh * nchunks;               // chunks over all halves: g = h * nchunks + c
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (warp == 0) tc::tmem_alloc(tmem_slot, TCOLS);
    if (tid == 0) {
        for (int i = 0; i < NBAR; ++i)
            tc::mbar_init(&bars[i], ((i >= B_RAWFREE && i < B_D) || i == B_TFREE) ? 128 : 1);
        tc::mbar_fence_init();
        *err = 0;
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp < 4) {
        // ---------------- epilogue: row me, y + acc per half ----------------
        const int me = warp * 32 + lane, row = row0 + me;
        float* qr = (p.tab ? p.tab[b] : p.one).Q + (long long)row * ldq;
        float* sr = scratch ? scratch + ((size_t)b * K + (size_t)(row < K ? row : 0)) * 256 : nullptr;
        const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
        // the addend y (this row of Q before the update; nothing writes it before the last half's epilogue) is loaded
        // one 32-column block ahead: the first before the products are done, each next one during the current one
        const bool addend = MODE != 1 && row < K;
        float4 yv[8], yn[8];
        auto load_y = [&](float4 (&y)[8], int col) {
#pragma unroll
            for (int i = 0; i < 8; ++i) y[i] = addend ? *reinterpret_cast<const float4*>(qr + col + 4 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
        };
        for (int h = 0; h < nh; ++h) {
            const int c0 = oc0 + h * N;
            load_y(yv, c0);
            const bool done = !*err && tc::mbar_wait_sleep(&bars[B_DONE], (uint32_t)(h & 1), 500);
            if (!__all_sync(0xffffffffu, done && !*err)) {   // per warp: tcgen05.ld needs the whole warp
                *err = 1;
                break;
            }
            tc::fence_after_sync();
            float* dst = (MODE == 1 || (nh > 1 && h + 1 < nh)) ? sr : qr + c0;   // an earlier half waits in scratch
            for (int cb = 0; cb < N / 32; ++cb) {
                if (cb + 1 < N / 32) load_y(yn, c0 + 32 * (cb + 1));
                float big[32], small[32];
                tc::tmem_ld32(tl + 32 * cb, big);
                tc::tmem_ld32(tl + 256 + 32 * cb, small);
                tc::tmem_wait_ld();
                if (MODE == 1 && row < K) {
#pragma unroll
                    for (int i = 0; i < 32; i += 4)
                        *reinterpret_cast<float4*>(dst + 32 * cb + i) =
                            make_float4(__fadd_rn(big[i], small[i]), __fadd_rn(big[i + 1], small[i + 1]),
                                        __fadd_rn(big[i + 2], small[i + 2]), __fadd_rn(big[i + 3], small[i + 3]));
                } else if (row < K) {
#pragma unroll
                    for (int i = 0; i < 32; i += 4) {
                        float4 y = yv[i / 4];
                        y.x = __fadd_rn(y.x, __fadd_rn(big[i], small[i]));
                        y.y = __fadd_rn(y.y, __fadd_rn(big[i + 1], small[i + 1]));
                        y.z = __fadd_rn(y.z, __fadd_rn(big[i + 2], small[i + 2]));
                        y.w = __fadd_rn(y.w, __fadd_rn(big[i + 3], small[i + 3]));
                        *reinterpret_cast<float4*>(dst + 32 * cb + i) = y;
                    }
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) yv[i] = yn[i];
            }
            if (nh > 1 && h + 1 < nh) {   // the next half's products may overwrite the accumulators
                tc::fence_before_sync();
                tc::mbar_arrive(&bars[B_TFREE]);
            }
        }
        if (MODE == 0 && nh > 1 && !*err && row < K) {   // every half's products have read this row: scratch goes in
            for (int c = 0; c < N; c += 4)
                *reinterpret_cast<float4*>(qr + c) = *reinterpret_cast<const float4*>(sr + c);
        }
    } else if (warp < 8) {
        // ---------------- convert: raw Q tile -> tf32 hi | lo, rows 16 i + t / 8, k-quad t % 8 ----------------
        const int t = tid - 128, aq = t & 7, am = t >> 3;
        for (int c = 0; c < total; ++c) {   // c: chunk over all halves
            const int st = c & 1;
            if (*err || !tc::mbar_wait(&bars[B_RAW + st], ring_parity(c))) {
                *err = 1;
                break;
            }
            const char* raw = RAW + st * YT;
            float4 v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = *reinterpret_cast<const float4*>(raw + 128 * (16 * i + am) + 16 * aq);
            // the next TMA load into this stage writes through the async proxy: order the generic reads above first
            tc::fence_async_smem();
            tc::mbar_arrive(&bars[B_RAWFREE + st]);
            if (c >= 2 && !tc::mbar_wait(&bars[B_FREE + st], ring_parity(c - 2))) {   // products of chunk c - 2 done
                *err = 1;
                break;
            }
            char* op = AOP + st * 2 * YT;
#pragma unroll
            for (int i = 0; i < 8; ++i) tc::store2_at(op, op + YT, tc::swz_off(16 * i + am, aq), v[i]);
            tc::fence_async_smem();
            tc::mbar_arrive(&bars[B_OP + st]);
        }
    } else if (warp == 8) {
        // ---------------- products ----------------
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_tf32(ROWS, N);
            bool ok = true;
            for (int g = 0; g < total; ++g) {
                const int st = g & 1, h = (nh > 1 && g >= nchunks) ? 1 : 0, c = g - h * nchunks;
                if (nh > 1 && c == 0 && h > 0) {   // the previous half's accumulators have been read
                    ok = !*err && tc::mbar_wait(&bars[B_TFREE], (uint32_t)((h - 1) & 1));
                    if (!ok) break;
                }
                ok = !*err && tc::mbar_wait(&bars[B_OP + st], ring_parity(g)) &&   // spin: the critical path
                     
                     tc::mbar_wait(&bars[B_D + st], ring_parity(g));
                if (!ok) break;
                tc::fence_after_sync();
                const uint32_t a = tc::smem_u32(AOP + st * 2 * YT), d = tc::smem_u32(DB + st * 2 * DPART);
#pragma unroll 1
                for (int k = 0; k < CH / 8; ++k) {
                    const uint64_t ahi = tc::sdesc_k128(a + 32 * k), alo = tc::sdesc_k128(a + YT + 32 * k);
                    const uint64_t dhi = tc::sdesc_k128(d + 32 * k), dlo = tc::sdesc_k128(d + N * 128 + 32 * k);
                    const uint32_t acc = (c > 0 || k > 0) ? 1u : 0u;
                    tc::mma_tf32(tmem, ahi, dhi, idesc, acc);
                    tc::mma_tf32(tmem + 256, ahi, dlo, idesc, acc);
                    tc::mma_tf32(tmem + 256, alo, dhi, idesc, 1u);
                }
                tc::mma_commit(&bars[B_FREE + st]);
                if (c == nchunks - 1) tc::mma_commit(&bars[B_DONE]);   // this half's products are done
            }
            if (!ok) {
                *err = 1;
                tc::mma_commit(&bars[B_FIN]);   // let issued products finish before TMEM is released
                tc::mbar_wait(&bars[B_FIN], 0u);
            }
        }
    } else {
        // ---------------- copies ----------------
        if (lane == 0) {
            const void* map = maps + ((size_t)b * TMAPS_PER_MATRIX + TMAP_Q) * 128;
            const char* img = img_all + (size_t)b * (MODE == 0   ? ns_dimg_bytes(n)
                                                     : MODE == 1 ? wcol_off(n / CH, n / CH)
                                                                 : band_img_bytes(ncontr));
            const uint32_t pbytes = (uint32_t)(N * 128);   // one half's rows of one part (hi or lo) of a D chunk
            tc::tmap_acquire(map);
            int n_raw[2] = {0, 0}, n_d[2] = {0, 0};
            bool ok = true;
            for (int g = 0; g < total; ++g) {
                const int st = g & 1, h = (nh > 1 && g >= nchunks) ? 1 : 0, c = g - h * nchunks;
                if (g >= 2) {
                    // raw tile g - 2 read by the convert warps; D chunk g - 2 read by its products
                    ok = !*err && tc::mbar_wait_sleep(&bars[B_RAWFREE + st], ring_parity(g - 2), 100) &&
                         tc::mbar_wait_sleep(&bars[B_FREE + st], ring_parity(g - 2), 100);
                    if (!ok) break;
                }
                tc::mbar_expect_tx(&bars[B_RAW + st], (uint32_t)YT);
                tc::tma_load_2d(RAW + st * YT, map, c * CH, row0, &bars[B_RAW + st]);
                ++n_raw[st];
                tc::mbar_expect_tx(&bars[B_D + st], 2 * pbytes);
                if (MODE == 0) {
                    const char* chunk = img + (size_t)c * 2 * n * 128 + (size_t)h * 2 * pbytes;   // hi rows, lo rows
                    tc::bulk_g2s(DB + st * 2 * DPART, chunk, 2 * pbytes, &bars[B_D + st]);
                } else if (MODE == 2) {   // chunk c of -T: hi rows, lo rows
                    tc::bulk_g2s(DB + st * 2 * DPART, img + (size_t)c * 2 * pbytes, 2 * pbytes, &bars[B_D + st]);
                } else {
                    // block column c of the W image: tiles j0 .. of its trailing list (hi), and the same in the lo list
                    const int NB = n / CH;
                    const char* hi = img + wcol_off(NB, c) + 2 * 4096 + (size_t)(j0 - c - 1) * 4096;
                    tc::bulk_g2s(DB + st * 2 * DPART, hi, pbytes, &bars[B_D + st]);
                    tc::bulk_g2s(DB + st * 2 * DPART + pbytes, hi + (size_t)(NB - 1 - c) * 4096, pbytes, &bars[B_D + st]);
                }
                ++n_d[st];
            }
            if (!ok) {
                *err = 1;
                for (int i = 0; i < 2; ++i) {   // let issued copies land before the shared memory is released
                    if (n_raw[i]) tc::mbar_wait(&bars[B_RAW + i], (uint32_t)((n_raw[i] - 1) & 1));
                    if (n_d[i]) tc::mbar_wait(&bars[B_D + i], (uint32_t)((n_d[i] - 1) & 1));
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (tid == 0 && *err) atomicOr(status, ERR_TIMEOUT);
    if (warp == 0) tc::tmem_dealloc(tmem, TCOLS);
}

template <int NH, int MODE>
static cudaError_t launch_k(PtrArg p, int K, int n, long long ldq, int B, const char* maps, const char* img,
                            float* scratch, int* status, int ncontr, int N, int j0, cudaStream_t st) {
    cudaError_t e = cudaFuncSetAttribute(k_ns_ws<NH, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    k_ns_ws<NH, MODE><<<dim3(cdiv(K, ROWS), B), NT, SMEM_BYTES, st>>>(p, K, n, ldq, maps, img, scratch, status, ncontr,
                                                                     N, j0);
    return cudaGetLastError();
}

cudaError_t launch_ns_ws(PtrArg p, int K, int n, long long ldq, int B, const float* D, const char* maps, char* img,
                         float* scratch, int* status, cudaStream_t st) {
    if (n > 512 || n % CH || (n > 256 && !scratch)) return cudaErrorInvalidValue;
    k_d_image<<<dim3(cdiv(n * n / 4, 256), B), 256, 0, st>>>(D, n, img);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    return n > 256 ? launch_k<2, 0>(p, K, n, ldq, B, maps, img, scratch, status, n, n / 2, 0, st)
                   : launch_k<1, 0>(p, K, n, ldq, B, maps, img, nullptr, status, n, n, 0, st);
}

cudaError_t launch_trsm_panel_product(PtrArg p, int K, int n, long long ldq, int B, int j0, int nbp, const char* maps,
                                      const char* W, float* scratch, int* status, cudaStream_t st) {
    if (n > 512 || n % CH || j0 < 1 || nbp < 1 || nbp > 8 || (j0 + nbp) * CH > n || !scratch) return cudaErrorInvalidValue;
    return launch_k<1, 1>(p, K, n, ldq, B, maps, W, scratch, status, j0 * CH, nbp * CH, j0, st);
}

cudaError_t launch_project(PtrArg p, int K, int n, long long ldq, int j, const char* maps, const char* img,
                           int* status, cudaStream_t st) {
    if (j < BLOCK_W || j % BLOCK_W || j + BLOCK_W > n || ldq < n) return cudaErrorInvalidValue;
    return launch_k<1, 2>(p, K, n, ldq, 1, maps, img, nullptr, status, j, BLOCK_W, j, st);
}

}  // namespace spq
