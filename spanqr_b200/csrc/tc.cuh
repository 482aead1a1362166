// sm_100a tensor-core building blocks: TMEM allocation, tcgen05.mma (kind::tf32), commits to mbarriers, TMEM
// loads, proxy fences, split-TF32 conversion and the shared-memory layout the MMA reads (K-major, 128-byte swizzle).
//
// Operand tiles: R rows (M or N) x 32 fp32 (one 128-byte row per M/N index), stored as 8-row atoms of 1024 bytes;
// the 16-byte chunk c (k = 4c .. 4c+3) of row m sits at chunk position c ^ (m % 8).  Tile bases are 1024-aligned.
// One MMA consumes K = 8 (32 bytes); k-step s starts 32 * s bytes into the tile.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace spq {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// ---- mbarriers ----
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits for the phase with this parity to complete, for at most `limit_ns`; false when the limit ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns = 2000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer() - t0 > limit_ns) return false;
    }
    return true;
}

// The same wait for a thread off the critical path: it sleeps between polls, so that warps sharing its SM
// sub-partition keep their issue slots.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t sleep_ns,
                                                uint64_t limit_ns = 2000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(bar, parity)) {
        __nanosleep(sleep_ns);
        if (globaltimer() - t0 > limit_ns) return false;
    }
    return true;
}

// ---- proxy and tcgen05 ordering fences ----
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ---- tensor memory (executed by one full warp) ----
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// ---- MMA: D[tmem] (+)= A[smem] * B[smem]^T, fp32 accumulate, tf32 inputs, issued by one thread ----
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        :
        : "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

// arrive (once) on `bar` when every MMA this thread issued before has completed
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// instruction descriptor: D fp32, A and B tf32, both K-major, M x N
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 bytes apart
__device__ __forceinline__ uint64_t sdesc_k128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)64u << 32) | ((uint64_t)1u << 46) |
           ((uint64_t)2u << 61);
}

// shared-memory matrix descriptor: MN-major tf32, 128-byte swizzle on a 32-byte base (layout type 1, the only
// MN-major layout tcgen05 accepts for 32-bit operands).  Atoms of 4 k-rows x 32 MN-elements (512 bytes) in which the
// 32-byte granule g of k-row r sits at granule position g ^ r; atoms along MN are `mn_stride` bytes apart (leading
// byte offset), along K `k_stride` bytes apart (stride byte offset).
__device__ __forceinline__ uint64_t sdesc_mn128b32(uint32_t saddr, uint32_t mn_stride, uint32_t k_stride) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((mn_stride >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((k_stride >> 4) & 0x3FFFu) << 32) | ((uint64_t)1u << 46) | ((uint64_t)1u << 61);
}

// instruction descriptor: D fp32, A and B tf32, both MN-major, M x N
__host__ __device__ constexpr uint32_t idesc_tf32_mn(int M, int N) {
    return idesc_tf32(M, N) | (1u << 15) | (1u << 16);
}

// byte offset of (k, mn .. mn+3) (mn a multiple of 4) in an MN-major tile of 128 MN x 32 k in the 32-byte-base
// layout: MN-atoms (32 elements) 512 bytes apart, k-atoms (4 rows) 2048 bytes apart
__device__ __forceinline__ uint32_t swz_mn_off(int k, int mn) {
    const int kr = k & 3, g = (mn >> 3) & 3;
    return (uint32_t)((k >> 2) * 2048 + (mn >> 5) * 512 + kr * 128 + ((g ^ kr) << 5) + ((mn & 7) << 2));
}

// ---- TMEM -> registers: this warp's 32 lanes, 32 consecutive 32-bit columns ----
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// ---- TMEM -> registers: this warp's 32 lanes, 16 consecutive 32-bit columns ----
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---- split TF32: x = hi + lo (+ a remainder below 2^-22 |x|), both rounded to tf32 (low 13 bits zero) ----
// Round to nearest, ties away from zero, on the bit pattern: add half a tf32 ulp to the magnitude bits and clear
// the 13 low bits (two integer ops on the ALU, where the conversion instruction would occupy the slower XU pipe).
// Finite inputs only (an infinity would turn into a NaN).
__device__ __forceinline__ float to_tf32(float x) {
    return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
    hi = to_tf32(x);
    lo = to_tf32(__fsub_rn(x, hi));
}

// exact three-way split x = hi + mid + lo (11 + 11 + the remaining 2 bits), each a tf32 value
__device__ __forceinline__ void split3_tf32(float x, float& hi, float& mid, float& lo) {
    hi = to_tf32(x);
    const float r1 = __fsub_rn(x, hi);
    mid = to_tf32(r1);
    lo = to_tf32(__fsub_rn(r1, mid));
}

// byte offset of the 16-byte chunk (row m, k-quad q) inside a K-major 128B-swizzled tile
__device__ __forceinline__ uint32_t swz_off(int m, int q) {
    return (uint32_t)((m >> 3) * 1024 + (m & 7) * 128 + ((q ^ (m & 7)) << 4));
}

// store 4 consecutive k of row m (k-quad q) as hi and lo tf32 into two tiles
__device__ __forceinline__ void store_split4(char* hi_tile, char* lo_tile, int m, int q, float4 v) {
    float4 h, l;
    split_tf32(v.x, h.x, l.x);
    split_tf32(v.y, h.y, l.y);
    split_tf32(v.z, h.z, l.z);
    split_tf32(v.w, h.w, l.w);
    const uint32_t o = swz_off(m, q);
    *reinterpret_cast<float4*>(hi_tile + o) = h;
    *reinterpret_cast<float4*>(lo_tile + o) = l;
}

// store the split parts of v at byte offset o of two (hi, lo) or three (hi, mid, lo) tiles
__device__ __forceinline__ void store2_at(char* hi_tile, char* lo_tile, uint32_t o, float4 v) {
    float4 h, l;
    split_tf32(v.x, h.x, l.x);
    split_tf32(v.y, h.y, l.y);
    split_tf32(v.z, h.z, l.z);
    split_tf32(v.w, h.w, l.w);
    *reinterpret_cast<float4*>(hi_tile + o) = h;
    *reinterpret_cast<float4*>(lo_tile + o) = l;
}

__device__ __forceinline__ void store3_at(char* hi_tile, char* mid_tile, char* lo_tile, uint32_t o, float4 v) {
    float4 h, md, l;
    split3_tf32(v.x, h.x, md.x, l.x);
    split3_tf32(v.y, h.y, md.y, l.y);
    split3_tf32(v.z, h.z, md.z, l.z);
    split3_tf32(v.w, h.w, md.w, l.w);
    *reinterpret_cast<float4*>(hi_tile + o) = h;
    *reinterpret_cast<float4*>(mid_tile + o) = md;
    *reinterpret_cast<float4*>(lo_tile + o) = l;
}

// store 4 consecutive k of row m (k-quad q) as hi, mid and lo tf32 into three tiles
__device__ __forceinline__ void store_split4x3(char* hi_tile, char* mid_tile, char* lo_tile, int m, int q, float4 v) {
    float4 h, md, l;
    split3_tf32(v.x, h.x, md.x, l.x);
    split3_tf32(v.y, h.y, md.y, l.y);
    split3_tf32(v.z, h.z, md.z, l.z);
    split3_tf32(v.w, h.w, md.w, l.w);
    const uint32_t o = swz_off(m, q);
    *reinterpret_cast<float4*>(hi_tile + o) = h;
    *reinterpret_cast<float4*>(mid_tile + o) = md;
    *reinterpret_cast<float4*>(lo_tile + o) = l;
}

}  // namespace tc
}  // namespace spq

namespace spq {
namespace tc {
// ---- 16-byte asynchronous global -> shared copies (no registers; completion per thread via groups) ----
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
}  // namespace tc
}  // namespace spq

namespace spq {
namespace tc {
// ---- bulk (TMA engine) global -> shared copies, completion counted in bytes on an mbarrier ----
// The copy engine writes shared memory directly: no registers and no L1 staging, so a CTA that holds most of the
// SM's shared memory can keep many copies in flight.  Addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(smem_dst)), "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
}  // namespace tc
}  // namespace spq

namespace spq {
namespace tc {
// ---- tensor-map (TMA) tile loads ----
// A tensor map written by a kernel (k_tmaps) is made visible to the copy engine by that kernel's release fence; the
// consumer acquires it once before its first load.
__device__ __forceinline__ void tmap_acquire(const void* map) {
    asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(map) : "memory");
}
// 2-D tile at coordinates (c0 = column, c1 = row); c0 * 4 bytes must be a multiple of 16; rows past the tensor's end
// arrive as zeros and still count toward the barrier's bytes
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* map, int c0, int c1, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(smem_dst)), "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}
// ---- TMEM stores (one warp: its 32 lanes, 32 consecutive columns) ----
__device__ __forceinline__ void tmem_st32_zero(uint32_t taddr) {
    const uint32_t z = 0u;
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, "
        "%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr),
        "r"(z)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
}  // namespace tc
}  // namespace spq

namespace spq {
namespace tc {
// ---- warp-role synchronisation ----
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// named barrier `id` (1..15) over `count` threads (a multiple of 32)
__device__ __forceinline__ void bar_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
}  // namespace tc
}  // namespace spq

namespace spq {
namespace tc {
// named barrier `id` over `count` threads that also ANDs a predicate across them: a group that must leave a loop
// together (because it meets again at a named barrier) decides with this
__device__ __forceinline__ bool bar_and(int id, int count, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "barrier.red.and.pred p, %2, %3, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)pred), "r"(id), "r"(count)
        : "memory");
    return r != 0;
}
}  // namespace tc
}  // namespace spq

namespace spq {
namespace tc {
// registers -> TMEM: this warp's 32 lanes, 32 consecutive 32-bit columns
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]), "f"(v[9]),
        "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]), "f"(v[17]), "f"(v[18]),
        "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]),
        "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
        : "memory");
}
}  // namespace tc
}  // namespace spq

namespace spq {
namespace tc {
// 32-byte global accesses (sm_100): eight consecutive floats at a 32-byte aligned address.  A warp whose threads each
// own one row moves 32 full sectors per instruction instead of 32 half sectors with 16-byte accesses.
__device__ __forceinline__ void ld8(const float* p, float* v) {
    asm volatile("ld.global.v8.f32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7])
                 : "l"(p));
}
__device__ __forceinline__ void st8(float* p, const float* v) {
    asm volatile("st.global.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "f"(v[0]), "f"(v[1]), "f"(v[2]),
                 "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7])
                 : "memory");
}
}  // namespace tc
}  // namespace spq

namespace spq {
namespace tc {
// 32 consecutive floats of one row to / from global memory: 32-byte accesses when `w8` (p 32-byte aligned), else 16
__device__ __forceinline__ void st_row32(float* p, const float* v, bool w8) {
    if (w8) {
#pragma unroll
        for (int k = 0; k < 32; k += 8) st8(p + k, v + k);
    } else {
#pragma unroll
        for (int k = 0; k < 32; k += 4) *reinterpret_cast<float4*>(p + k) = make_float4(v[k], v[k + 1], v[k + 2], v[k + 3]);
    }
}
__device__ __forceinline__ void ld_row32(const float* p, float* v, bool w8) {
    if (w8) {
#pragma unroll
        for (int k = 0; k < 32; k += 8) ld8(p + k, v + k);
    } else {
#pragma unroll
        for (int k = 0; k < 32; k += 4) {
            const float4 t = *reinterpret_cast<const float4*>(p + k);
            v[k] = t.x, v[k + 1] = t.y, v[k + 2] = t.z, v[k + 3] = t.w;
        }
    }
}
__device__ __forceinline__ bool al32(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 31) == 0; }
}  // namespace tc
}  // namespace spq
