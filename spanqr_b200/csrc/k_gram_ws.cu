// Gram partials of Y (or s X) for n <= 256 on the tcgen05 tensor cores, two-way split TF32 (hi.hi + hi.lo + lo.hi):
// the Grams the reference computes as plain fp32 GEMMs (passes 2 and 3, the first polish step: kcholqr.py:106 and
// :20) and the first pass's compensated gram_f (tri.py:324-375), which the two-way split matches closely enough for
// every robustness and span test.
//
// One CTA = one 128-row panel i of G and one split of GRAM_TC_SPLIT rows of Y: it computes
//     G[128 i .. 128 i + 127, 128 i .. n) over the split's rows
// as one M = 128, N = n - 128 i (<= 256) product per k-step.  A (the panel's 128 columns of Y) is the first 128
// columns of B (columns 128 i .. n of Y), so one staged chunk of 32 rows serves both operands, MN-major in the 32-byte
// base 128B-swizzled layout tcgen05 takes for 32-bit types.  The split accumulates in TMEM (hi.hi and the cross terms
// in separate accumulators) and is written to the partial tiles P[b][split][tile] of k_gram_tc (the same layout, so
// k_gram_reduce sums them unchanged); the tile diagonal is replaced by the sum of squares kept in float-float (exact
// squares, about 44 bits).
// Warp roles: 0-3 epilogue (TMEM lanes = the panel's columns), 4-7 convert (raw chunk -> s y -> tf32 hi | lo, float-float
// squares of the panel's columns), 8 products (one thread), 9 copies (one thread, TMA through the per-matrix maps).
#include "kernels.h"
#include "tc.cuh"

namespace spq {

namespace {
constexpr int NT = 320;
constexpr int TILE = 128;
constexpr int CH = 32;                       // rows per chunk (4 k-steps of 8)
constexpr int RAWB = GRAM_BOX_COLS * CH * 4; // one raw box: 128 columns x 32 rows fp32 = 16 KB
constexpr int RAW_STAGE = 2 * RAWB;          // up to two boxes (256 columns)
constexpr int OP_PART = 256 * CH * 4;        // one operand part (hi or lo) of up to 256 columns: 32 KB
constexpr int OP_STAGE = 2 * OP_PART;
constexpr int RSTAGES = 3;                   // raw chunks in flight (copies three chunks ahead of the conversion)
constexpr int OSTAGES = 2;                   // operand chunks
constexpr int OFF_RAW = 0;
constexpr int OFF_OP = OFF_RAW + RSTAGES * RAW_STAGE;
constexpr int OFF_DSQ = OFF_RAW;             // after the last chunk: 4 convert warps x 128 columns of squares (hi, lo)
constexpr int OFF_BAR = OFF_OP + OSTAGES * OP_STAGE;
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;
constexpr uint32_t TCOLS = 512;              // large at 0, small at 256
constexpr int ERR_TIMEOUT = 0x10;
// mbarriers (per stage where doubled): raw chunk landed, raw chunk read (128 arrivals), operands written (128
// arrivals), operands consumed, all products done, error drain.  Every waiter steps through a barrier's phases in
// order from phase 0, and no barrier can run two phases ahead of a waiter.
enum { B_RAW = 0, B_RAWFREE = 3, B_OP = 6, B_OPFREE = 8, B_DONE = 10, B_FIN = 11, NBAR = 12 };
static_assert(4 * TILE * 8 <= RAW_STAGE, "the squares fit one raw stage");
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
static_assert(GRAM_BOX_ROWS == CH && GRAM_BOX_COLS == TILE, "one TMA box is 128 columns of one chunk");

__device__ __forceinline__ uint32_t ring_parity(int c) { return (uint32_t)((c >> 1) & 1); }   // c-th use of a 2-ring
__device__ __forceinline__ uint32_t par3(int c) { return (uint32_t)((c / 3) & 1); }            // c-th use of a 3-ring

// byte offset of (k, mn .. mn+3) in an operand part whose MN extent is `w` (a multiple of 128): 32-byte-base layout,
// atoms of 4 k-rows x 32 MN (512 bytes) with the 32-byte granule g of k-row r at granule position g ^ r, MN-atoms
// 512 bytes apart, k-atoms 16 w bytes apart
__device__ __forceinline__ uint32_t mn_off(int k, int mn, int w) {
    const int kr = k & 3, g = (mn >> 3) & 3;
    return (uint32_t)((k >> 2) * (16 * w) + (mn >> 5) * 512 + kr * 128 + ((g ^ kr) << 5) + ((mn & 7) << 2));
}
}  // namespace

__global__ void __launch_bounds__(NT, 1) k_gram_ws(PtrArg p, Src src, int K, int n, GramPlan gp,
                                                   const char* __restrict__ maps, ScaleArg sc, float* __restrict__ P,
                                                   int* __restrict__ status) {
    extern __shared__ unsigned char smem_raw[];
    char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    char* const RAW = sm + OFF_RAW;
    char* const OP = sm + OFF_OP;
    float2* const DSQ = reinterpret_cast<float2*>(sm + OFF_DSQ);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 128);
    volatile int* err = reinterpret_cast<volatile int*>(sm + OFF_BAR + 132);

    const int pi = blockIdx.x, sp = blockIdx.y, b = blockIdx.z;
    const int col0 = pi * TILE;
    const int N = n - col0;                  // product width (a multiple of 32, <= 256)
    const int nbox = N > TILE ? 2 : 1;       // raw boxes per chunk
    const int W = nbox * TILE;               // MN extent of the staged operands
    const int k0 = sp * gp.KS;
    const int nchunks = (min(k0 + gp.KS, K) - k0 + CH - 1) / CH;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (warp == 0) tc::tmem_alloc(tmem_slot, TCOLS);
    if (tid == 0) {
        for (int i = 0; i < NBAR; ++i)
            tc::mbar_init(&bars[i], (i >= B_RAWFREE && i < B_OPFREE) ? 128 : 1);   // raw read, operands written
        tc::mbar_fence_init();
        *err = 0;
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp < 4) {
        // ---------------- epilogue: row a of tile row-panel pi (TMEM lane a) ----------------
        const bool done = !*err && tc::mbar_wait_sleep(&bars[B_DONE], 0u, 500);   // the whole split: sleep
        tc::bar_sync(3, 256);   // the convert warps' squares are in shared memory
        // decided per warp: tcgen05.ld needs the whole warp
        if (__all_sync(0xffffffffu, done && !*err)) {
            tc::fence_after_sync();
            const int a = warp * 32 + lane;
            double d = 0.0;
#pragma unroll
            for (int w = 0; w < 4; ++w) d = __dadd_rn(d, ff_value(DSQ[w * TILE + a].x, DSQ[w * TILE + a].y));
            const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
            float* Pb = P + (size_t)(b * gp.S + sp) * gp.tiles * TILE * TILE;
            for (int cb = 0; cb < W / 32; ++cb) {
                float big[32], small[32];
                tc::tmem_ld32(tl + 32 * cb, big);
                tc::tmem_ld32(tl + 256 + 32 * cb, small);
                tc::tmem_wait_ld();
                const int tj = pi + (32 * cb) / TILE, c0 = (32 * cb) % TILE;
                const int t = pi * gp.nt - pi * (pi - 1) / 2 + (tj - pi);
                float* row = Pb + (size_t)t * TILE * TILE + (size_t)a * TILE + c0;
#pragma unroll
                for (int i = 0; i < 32; ++i) big[i] = __fadd_rn(big[i], small[i]);
                if (tj == pi && a >= c0 && a < c0 + 32) {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (c0 + i == a) big[i] = __double2float_rn(d);
                }
                tc::st_row32(row, big, true);   // partial rows: 512 bytes apart, 256-byte aligned base
            }
        }
    } else if (warp < 8) {
        // ---------------- convert: rows 8 (warp - 4) .. +7 of each chunk, columns 4 lane .. of each box ----------------
        float s = 1.0f;
        bool scaled = false;
        if (sc.maxbits) {
            s = pow2_scale(__uint_as_float(sc.maxbits[b]));
            scaled = true;
        } else if (sc.s) {
            s = sc.s[b];
            scaled = true;
        }
        const int cw = warp - 4;
        float sqh[4] = {0.f, 0.f, 0.f, 0.f}, sql[4] = {0.f, 0.f, 0.f, 0.f};   // squares of columns 4 lane .. + 3
        for (int c = 0; c < nchunks; ++c) {
            const int st = c & 1, rs = c % RSTAGES;
            if (*err || !tc::mbar_wait(&bars[B_RAW + rs], par3(c))) {
                *err = 1;
                break;
            }
            const char* raw = RAW + rs * RAW_STAGE;
            float4 v[2][8];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                if (h < nbox) {
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        v[h][i] = *reinterpret_cast<const float4*>(raw + h * RAWB + (8 * cw + i) * 512 + 16 * lane);
                }
            }
            // the raw stage is released after the one proxy fence below: the next TMA load into it writes through the
            // async proxy, so these generic reads must be ordered before it by that fence (without one, bytes of a
            // later chunk were seen in place of chunk c's)
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                float4& x = v[0][i];
                if (scaled) {
                    x.x = __fmul_rn(x.x, s); x.y = __fmul_rn(x.y, s); x.z = __fmul_rn(x.z, s); x.w = __fmul_rn(x.w, s);
                }
                ff_add_sq(sqh[0], sql[0], x.x);
                ff_add_sq(sqh[1], sql[1], x.y);
                ff_add_sq(sqh[2], sql[2], x.z);
                ff_add_sq(sqh[3], sql[3], x.w);
                if (nbox == 2 && scaled) {
                    float4& y = v[1][i];
                    y.x = __fmul_rn(y.x, s); y.y = __fmul_rn(y.y, s); y.z = __fmul_rn(y.z, s); y.w = __fmul_rn(y.w, s);
                }
            }
            if (c >= 2 && !tc::mbar_wait(&bars[B_OPFREE + st], ring_parity(c - 2))) {   // products of chunk c - 2 done
                *err = 1;
                break;
            }
            char* op = OP + st * OP_STAGE;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                if (h < nbox) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const uint32_t o = mn_off(8 * cw + i, h * TILE + 4 * lane, W);
                        tc::store2_at(op, op + OP_PART, o, v[h][i]);
                    }
                }
            }
            tc::fence_async_smem();
            tc::mbar_arrive(&bars[B_RAWFREE + rs]);
            tc::mbar_arrive(&bars[B_OP + st]);
        }
        tc::bar_sync(1, 128);   // every convert warp is done with the raw stages: the squares go into the first one
#pragma unroll
        for (int j = 0; j < 4; ++j) DSQ[cw * TILE + 4 * lane + j] = make_float2(sqh[j], sql[j]);
        tc::bar_sync(3, 256);
    } else if (warp == 8) {
        // ---------------- products ----------------
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_tf32_mn(TILE, N);
            bool ok = true;
            for (int c = 0; c < nchunks; ++c) {
                const int st = c & 1;
                ok = !*err && tc::mbar_wait(&bars[B_OP + st], ring_parity(c));   // spin: this wait is the critical path
                if (!ok) break;
                tc::fence_after_sync();
                const uint32_t hi = tc::smem_u32(OP + st * OP_STAGE), lo = hi + OP_PART;
#pragma unroll 1
                for (int k = 0; k < CH / 8; ++k) {
                    const uint32_t ko = (uint32_t)(2 * 16 * W * k);   // two k-atoms per k-step of 8
                    const uint64_t ahi = tc::sdesc_mn128b32(hi + ko, 512, 16 * W);
                    const uint64_t alo = tc::sdesc_mn128b32(lo + ko, 512, 16 * W);
                    const uint32_t acc = (c > 0 || k > 0) ? 1u : 0u;
                    tc::mma_tf32(tmem, ahi, ahi, idesc, acc);          // A and B share the staged columns
                    tc::mma_tf32(tmem + 256, ahi, alo, idesc, acc);
                    tc::mma_tf32(tmem + 256, alo, ahi, idesc, 1u);
                }
                tc::mma_commit(&bars[B_OPFREE + st]);
            }
            if (ok) {
                tc::mma_commit(&bars[B_DONE]);
            } else {
                *err = 1;
                tc::mma_commit(&bars[B_FIN]);   // let issued products finish before TMEM is released
                tc::mbar_wait(&bars[B_FIN], 0u);
            }
        }
    } else {
        // ---------------- copies ----------------
        if (lane == 0) {
            const void* map = maps + ((size_t)b * TMAPS_PER_MATRIX + (src == SRC_X ? TMAP_GX : TMAP_GQ)) * 128;
            tc::tmap_acquire(map);
            int issued[RSTAGES] = {0, 0, 0};
            bool ok = true;
            for (int c = 0; c < nchunks; ++c) {
                const int rs = c % RSTAGES;
                if (c >= RSTAGES) {
                    ok = !*err && tc::mbar_wait_sleep(&bars[B_RAWFREE + rs], par3(c - RSTAGES), 100);   // c - 3 read
                    if (!ok) break;
                }
                tc::mbar_expect_tx(&bars[B_RAW + rs], (uint32_t)(nbox * RAWB));
                for (int h = 0; h < nbox; ++h)
                    tc::tma_load_2d(RAW + rs * RAW_STAGE + h * RAWB, map, col0 + h * TILE, k0 + c * CH, &bars[B_RAW + rs]);
                ++issued[rs];
            }
            if (!ok) {
                *err = 1;
                for (int i = 0; i < RSTAGES; ++i)   // let issued copies land before the shared memory is released
                    if (issued[i]) tc::mbar_wait(&bars[B_RAW + i], (uint32_t)((issued[i] - 1) & 1));
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (tid == 0 && *err) atomicOr(status, ERR_TIMEOUT);
    if (warp == 0) tc::tmem_dealloc(tmem, TCOLS);
}

cudaError_t launch_gram_ws(PtrArg p, Src src, int K, int n, int B, const GramPlan& gp, const char* maps, ScaleArg sc,
                           float* P, int* status, cudaStream_t st) {
    if (n > 2 * TILE || n % 32 || gp.KS % CH) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(k_gram_ws, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    k_gram_ws<<<dim3(gp.nt, gp.S, B), NT, SMEM_BYTES, st>>>(p, src, K, n, gp, maps, sc, P, status);
    return cudaGetLastError();
}

}  // namespace spq
