// tcgen05 grouped GEMM for segment_mm / gather_mm (replaces the serial
// src/ported.mojo:773-804 and the per-row src/ported.mojo:1089-1130).
//
// A persistent, warp-specialised kernel, one CTA per SM walking 128-row x
// BN-column tiles (a tile never crosses a segment).  A rows and the segment's
// K-major B block arrive in 128-byte K slices (32 fp32 or 64 bf16 values,
// SWIZZLE_128B layout) through two rings of their own: kStagesA slices of A
// (a DRAM stream, so the deeper ring) and kStagesB slices of B (a block that
// stays in L2).  Warp 0 issues B's TMA loads; warp 6 issues A's (segment_mm),
// or, for gather_mm, warps 6-9 gather each tile's A rows through the row
// permutation with 16-byte cp.async copies straight into the swizzled stage
// (no materialised copy of the gathered rows).  Warp 1 (one elected thread)
// issues tcgen05.mma (kind::tf32 for fp32 inputs, kind::f16 with bf16 for bf16
// inputs) into one of two 128 x BN fp32 accumulators in tensor memory; warps
// 2-5 read the other accumulator back with tcgen05.ld (each warp its 32-lane
// quarter) into a swizzled shared-memory staging box and write it with a TMA
// tile store (segment_mm rows inside the segment), or store the rows
// themselves (a segment's last partial tile; gather_mm's rows, scattered
// through `perm`), while the next tile's loads and MMAs run.
//
// Every mbarrier wait is bounded (kTimeoutNs of %globaltimer); the first to
// expire records an error code in g_bgl_tc_error and raises a CTA-wide abort
// flag that ends every role's loop; the producers then wait (bounded) for the
// loads they issued and the MMA thread for the MMAs it issued, so no copy or
// MMA is in flight when the tensor memory is freed and the CTA exits.
#include <cuda.h>
#include <cuda_bf16.h>

#include <mutex>

#include "grouped_mm.cuh"

namespace bgl {

__device__ int g_bgl_tc_error = 0;

namespace {

// Ring depths and epilogue width (build-time tuning knobs; shared memory:
// stagesA x 16 KB + stagesB x BN x 128 B + epilogue warps x 4 KB <= 227 KB).
#ifndef BGL_GMM_STAGES_A
#define BGL_GMM_STAGES_A 6
#endif
#ifndef BGL_GMM_STAGES_B
#define BGL_GMM_STAGES_B 3
#endif
#ifndef BGL_GMM_EPI_WARPS
#define BGL_GMM_EPI_WARPS 4
#endif
constexpr int kBM = 128;
constexpr int kStagesA = BGL_GMM_STAGES_A;  // A slices in flight (DRAM latency)
constexpr int kStagesB = BGL_GMM_STAGES_B;  // B slices in flight (L2 latency)
constexpr int kEpiWarps = BGL_GMM_EPI_WARPS;  // 4 or 8: one or two warps per TMEM lane quarter
static_assert(kEpiWarps == 4 || kEpiWarps == 8, "epilogue warps: 4 or 8");
constexpr int kStageRowBytes = 128;  // epilogue staging: 32 fp32 (or bf16 pairs) per row
constexpr int kABytes = kBM * 128;   // one A slice: 128 rows x 128 bytes
constexpr unsigned long long kTimeoutNs = 2000000000ull;  // 2 s per wait

// Warp roles.
constexpr int kWarpB = 0, kWarpMma = 1, kWarpEpi0 = 2, kWarpA0 = kWarpEpi0 + kEpiWarps;
__host__ __device__ constexpr int threads_for(bool gather) { return 32 * (kWarpA0 + (gather ? 4 : 1)); }

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long now_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: false if the phase has not completed within kTimeoutNs (the
// error word and the CTA's abort flag are then set) or if another role of the
// CTA has aborted (abort == nullptr: wait regardless of the flag).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int code,
                                          volatile int *abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = now_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (abort && *abort) return false;
        if (now_ns() - t0 > kTimeoutNs) {
            atomicCAS(&g_bgl_tc_error, 0, code);
            if (abort) *abort = 1;
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int32_t c0, int32_t c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cta.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

// 16-byte cp.async into shared memory; src_bytes = 0 writes zeros (a row past
// the segment, or K past d1) without reading.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
                 "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// Makes this thread's completed generic-proxy shared-memory writes (cp.async)
// visible to the async proxy that tcgen05.mma reads its operands through.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// TMA tile store of a staged (SWIZZLE_128B) box; the bulk-group waits let the
// staging buffer be rewritten once the store has read it.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *src, int32_t c0,
                                             int32_t c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(c0), "r"(c1), "r"(smem_u32(src))
        : "memory");
}
__device__ __forceinline__ void bulk_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// K-major, SWIZZLE_128B shared-memory matrix descriptor: rows of 128 bytes,
// 8-row groups 1024 bytes apart (SBO), LBO unused (1), version 1, layout 2.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

template <bool BF16>
__device__ __forceinline__ void mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                    uint32_t idesc, uint32_t accumulate) {
    if (BF16) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(
                tmem_d),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(
                tmem_d),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
    }
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// 16 consecutive fp32 columns of the warp's 32 TMEM lanes (one row a thread).
__device__ __forceinline__ void tmem_ld16(uint32_t addr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(addr));
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

struct TcArgs {
    void *out;
    const void *a;        // gather_mm: the A rows, read through perm
    int64_t a_row_bytes;  // gather_mm: bytes of one A row (d1 * element size)
    const int64_t *seg_off;
    const int64_t *tile_off;
    const int32_t *perm;  // gather_mm: output row of permuted row i
    int64_t r;
    int64_t n;
    int32_t d1;
    int32_t d2;
    int32_t bn;      // N columns of one CTA tile (multiple of 16, <= 256)
    int32_t kb;      // number of 128-byte K slices
    int32_t nbn;     // column tiles per row tile
};

// Instruction descriptor: fp32 accumulator, A/B format (TF32 = 2, BF16 = 1),
// both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t instr_desc(bool bf16, int n) {
    return (1u << 4) | ((bf16 ? 1u : 2u) << 7) | ((bf16 ? 1u : 2u) << 10) |
           ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

// Row tile `tile` -> (segment, first row, end of the segment's rows).
__device__ __forceinline__ void tile_rows(const TcArgs &args, int64_t tile, int64_t &rel,
                                          int64_t &row0, int64_t &row_end) {
    int64_t lo = 0, hi = args.r;
    while (lo < hi) {
        int64_t mid = (lo + hi + 1) >> 1;
        if (args.tile_off[mid] <= tile) lo = mid; else hi = mid - 1;
    }
    rel = lo;
    row0 = args.seg_off[rel] + (tile - args.tile_off[rel]) * kBM;
    row_end = args.seg_off[rel + 1];
}

template <bool BF16, bool GATHER>
__global__ void __launch_bounds__(threads_for(GATHER), 1)
    k_gmm_tc(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
             const __grid_constant__ CUtensorMap map_out, const TcArgs args) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    constexpr int SA = kStagesA;
    constexpr int kLag = SA - 2;  // cp.async groups a gather thread keeps open
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // this CTA's (row tile, column tile) pairs w = row_tile * nbn + column_tile:
    // blockIdx.x, blockIdx.x + gridDim.x, ... below the pair count
    const int64_t work = args.tile_off[args.r] * args.nbn;
    const uint32_t b_bytes = (uint32_t)args.bn * 128;  // one B slice
    const uint32_t b_region = kStagesB * b_bytes;
    // stage buffers, each 1024-byte aligned (the SWIZZLE_128B atom)
    uintptr_t base = (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023);
    unsigned char *sa = reinterpret_cast<unsigned char *>(base);
    unsigned char *sb = sa + SA * kABytes;
    // epilogue staging: per epilogue warp two buffers of 32 rows x 128 bytes
    uint4 *staging = reinterpret_cast<uint4 *>(sb + b_region);
    uint64_t *a_full =
        reinterpret_cast<uint64_t *>(sb + b_region + kEpiWarps * 2 * kStageRowBytes * 32);
    uint64_t *a_empty = a_full + SA;
    uint64_t *b_full = a_empty + SA;
    uint64_t *b_empty = b_full + kStagesB;
    uint64_t *acc_full = b_empty + kStagesB;  // [2]: accumulator b holds a finished tile
    uint64_t *acc_empty = acc_full + 2;       // [2]: the epilogue has read accumulator b
    uint64_t *mma_done = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    if (threadIdx.x == 0) {
        for (int s = 0; s < SA; ++s) {
            // gather: one arrive per gather thread once its copies have landed
            mbar_init(&a_full[s], GATHER ? 128 : 1);
            mbar_init(&a_empty[s], 1);
        }
        for (int s = 0; s < kStagesB; ++s) {
            mbar_init(&b_full[s], 1);
            mbar_init(&b_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], kEpiWarps);  // one arrive per epilogue warp
        }
        mbar_init(mma_done, 1);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    const uint32_t acc_cols = args.bn <= 32 ? 32 : args.bn <= 64 ? 64 : args.bn <= 128 ? 128 : 256;
    if (warp == kWarpMma) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(2 * acc_cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    const int kb_n = args.kb;

    if (warp == kWarpB) {
        if (lane == 0) {
            // B producer: slice `it` counts across this CTA's tiles
            int64_t it = 0;
            bool ok = true;
            for (int64_t w = blockIdx.x; w < work && ok; w += gridDim.x) {
                int64_t rel, row0, row_end;
                tile_rows(args, w / args.nbn, rel, row0, row_end);
                const int32_t nb = (int32_t)(w % args.nbn);
                for (int kb = 0; kb < kb_n; ++kb, ++it) {
                    const int s = (int)(it % kStagesB);
                    if (it >= kStagesB &&
                        !(ok = mbar_wait(&b_empty[s], (uint32_t)((it / kStagesB) - 1) & 1, 1, abort)))
                        break;
                    mbar_arrive_expect_tx(&b_full[s], b_bytes);
                    tma_load_2d(sb + s * b_bytes, &map_b, &b_full[s], kb * (BF16 ? 64 : 32),
                                (int32_t)(rel * args.d2 + (int64_t)nb * args.bn));
                }
            }
            // the last issued loads (at most one per stage) have landed before exit
            for (int64_t j = (it > kStagesB ? it - kStagesB : 0); j < it; ++j)
                mbar_wait(&b_full[j % kStagesB], (uint32_t)(j / kStagesB) & 1, 2, nullptr);
        }
    } else if (!GATHER && warp == kWarpA0) {
        if (lane == 0) {
            // A producer (segment_mm): TMA tile loads of 128 rows
            int64_t it = 0;
            bool ok = true;
            for (int64_t w = blockIdx.x; w < work && ok; w += gridDim.x) {
                int64_t rel, row0, row_end;
                tile_rows(args, w / args.nbn, rel, row0, row_end);
                for (int kb = 0; kb < kb_n; ++kb, ++it) {
                    const int s = (int)(it % SA);
                    if (it >= SA && !(ok = mbar_wait(&a_empty[s], (uint32_t)((it / SA) - 1) & 1, 1, abort)))
                        break;
                    mbar_arrive_expect_tx(&a_full[s], kABytes);
                    tma_load_2d(sa + s * kABytes, &map_a, &a_full[s], kb * (BF16 ? 64 : 32),
                                (int32_t)row0);
                }
            }
            for (int64_t j = (it > SA ? it - SA : 0); j < it; ++j)
                mbar_wait(&a_full[j % SA], (uint32_t)(j / SA) & 1, 2, nullptr);
        }
    } else if (GATHER && warp >= kWarpA0) {
        // A producers (gather_mm): thread g copies 16-byte chunk c = g % 8 of
        // the 128-byte K slice for rows rsub + 16 i (i < 8), rsub = g / 8, so
        // each warp instruction moves 4 whole 128-byte row slices.  Its copies
        // of slice `it` form one cp.async group; once a group is kLag (ring
        // depth - 2) groups old it has landed, and the thread publishes it to the async
        // proxy and arrives on the stage's barrier.
        const int g = threadIdx.x - kWarpA0 * 32;
        const int c = g & 7, rsub = g >> 3;
        const uint32_t sw = (uint32_t)((c ^ (rsub & 7)) << 4);  // SWIZZLE_128B: chunk ^ (row & 7)
        const char *a = static_cast<const char *>(args.a);
        int64_t it = 0;
        bool ok = true;
        for (int64_t w = blockIdx.x; w < work && ok; w += gridDim.x) {
            int64_t rel, row0, row_end;
            tile_rows(args, w / args.nbn, rel, row0, row_end);
            const char *src[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int64_t row = row0 + rsub + 16 * i;
                src[i] = row < row_end ? a + (int64_t)args.perm[row] * args.a_row_bytes + c * 16
                                       : nullptr;
            }
            for (int kb = 0; kb < kb_n; ++kb, ++it) {
                const int s = (int)(it % SA);
                if (it >= SA &&
                    !(ok = mbar_wait(&a_empty[s], (uint32_t)((it / SA) - 1) & 1, 1, abort)))
                    break;
                const int64_t koff = (int64_t)kb * 128;
                const bool kin = koff + c * 16 < args.a_row_bytes;
                const uint32_t dst = smem_u32(sa + s * kABytes) + (uint32_t)rsub * 128 + sw;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const bool live = src[i] != nullptr && kin;
                    cp_async16(dst + (uint32_t)i * 16 * 128, live ? src[i] + koff : a,
                               live ? 16u : 0u);
                }
                cp_async_commit();
                if (it >= kLag) {
                    cp_async_wait<kLag>();
                    fence_proxy_async_smem();
                    mbar_arrive(&a_full[(it - kLag) % SA]);
                }
            }
        }
        // every copy issued above has landed before the CTA moves on; stages
        // not yet published are published (an aborted CTA skips that)
        cp_async_wait<0>();
        fence_proxy_async_smem();
        if (ok)
            for (int64_t j = (it > kLag ? it - kLag : 0); j < it; ++j)
                mbar_arrive(&a_full[j % SA]);
    } else if (warp == kWarpMma) {
        if (lane == 0) {
            // MMA issuer: tile t accumulates into accumulator t & 1
            const uint32_t idesc = instr_desc(BF16, args.bn);
            int64_t it = 0, t = 0;
            bool ok = true;
            for (int64_t w = blockIdx.x; w < work && ok; w += gridDim.x, ++t) {
                const int b = (int)(t & 1);
                if (t >= 2 && !(ok = mbar_wait(&acc_empty[b], (uint32_t)((t >> 1) - 1) & 1, 5, abort)))
                    break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t dacc = tmem + (uint32_t)b * acc_cols;
                for (int kb = 0; kb < kb_n; ++kb, ++it) {
                    const int s_a = (int)(it % SA), s_b = (int)(it % kStagesB);
                    if (!(ok = mbar_wait(&a_full[s_a], (uint32_t)(it / SA) & 1, 3, abort))) break;
                    if (!(ok = mbar_wait(&b_full[s_b], (uint32_t)(it / kStagesB) & 1, 3, abort))) break;
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint64_t ad = smem_desc(smem_u32(sa + s_a * kABytes));
                    const uint64_t bd = smem_desc(smem_u32(sb + s_b * b_bytes));
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)  // 4 MMAs of 32 bytes of K per 128-byte slice
                        mma<BF16>(dacc, ad + kk * 2, bd + kk * 2, idesc, (kb | kk) != 0);
                    mma_commit(&a_empty[s_a]);
                    mma_commit(&b_empty[s_b]);
                }
                if (ok) mma_commit(&acc_full[b]);
            }
            // every MMA issued above has completed before the memory is freed
            mma_commit(mma_done);
            mbar_wait(mma_done, 0, 6, nullptr);
        }
    } else if (warp >= kWarpEpi0 && warp < kWarpEpi0 + kEpiWarps) {
        // epilogue: warp w reads TMEM lanes [32 (w % 4), 32 (w % 4) + 32); with
        // 8 epilogue warps the two warps of a lane quarter take alternate
        // chunks.  A chunk is CW columns, 128 bytes of each of the warp's 32
        // rows: each thread writes its row into a staging buffer (16-byte
        // pieces XOR-swizzled by row -- the SWIZZLE_128B layout, so neither
        // side conflicts on banks); when all 32 rows lie inside the segment
        // (segment_mm) one TMA store writes the 32 x CW box, otherwise the
        // warp stores the rows itself, 4 rows of 128 bytes per instruction
        // (scattered through perm for gather_mm).  Two staging buffers
        // alternate; a buffer is rewritten once the store that read it is done.
        const int q = warp & 3;
        const int part = (warp - kWarpEpi0) >> 2, parts = kEpiWarps >> 2;
        constexpr int CW = BF16 ? 64 : 32;
        uint4 *stg_base = staging + (warp - kWarpEpi0) * 2 * 32 * 8;
        int64_t t = 0;
        uint32_t chunk = 0;
        int last_commit = -1;  // staging buffer of this warp's latest TMA store
        for (int64_t w = blockIdx.x; w < work; w += gridDim.x, ++t) {
            const int b = (int)(t & 1);
            if (!mbar_wait(&acc_full[b], (uint32_t)(t >> 1) & 1, 4, abort)) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            int64_t rel, row0, row_end;
            tile_rows(args, w / args.nbn, rel, row0, row_end);
            const int32_t col0 = (int32_t)(w % args.nbn) * args.bn;
            const int64_t row = row0 + q * 32 + lane;
            const bool live = row < row_end;
            const int64_t orow = live ? (args.perm ? (int64_t)args.perm[row] : row) : 0;
            const bool whole = !GATHER && row0 + q * 32 + 32 <= row_end;  // warp-uniform
            const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)b * acc_cols;
            for (int c = CW * part; c < args.bn; c += CW * parts, ++chunk) {
                const int buf = (int)(chunk & 1);
                uint4 *stg = stg_base + buf * 32 * 8;
                if (lane == 0) {
                    if (last_commit == buf) bulk_wait_read<0>();
                    else bulk_wait_read<1>();
                }
                __syncwarp();
                if (BF16) {
                    uint32_t v[64];
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        tmem_ld16(taddr + (uint32_t)(c + 16 * k),
                                  *reinterpret_cast<uint32_t(*)[16]>(&v[16 * k]));
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        uint32_t o[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(v[8 * j + 2 * i]),
                                                                     __uint_as_float(v[8 * j + 2 * i + 1]));
                            o[i] = *reinterpret_cast<uint32_t *>(&h);
                        }
                        stg[lane * 8 + (j ^ (lane & 7))] = make_uint4(o[0], o[1], o[2], o[3]);
                    }
                } else {
                    uint32_t v[32];
                    tmem_ld16(taddr + (uint32_t)c, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
                    tmem_ld16(taddr + (uint32_t)c + 16, *reinterpret_cast<uint32_t(*)[16]>(&v[16]));
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        stg[lane * 8 + (j ^ (lane & 7))] =
                            make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                }
                if (whole) {
                    fence_proxy_async_smem();  // staged rows visible to the TMA unit
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&map_out, stg, col0 + c, (int32_t)(row0 + q * 32));
                        bulk_commit();
                        last_commit = buf;
                    }
                } else {
                    __syncwarp();
#pragma unroll
                    for (int pass = 0; pass < 8; ++pass) {
                        const int rr = pass * 4 + (lane >> 3), j = lane & 7;
                        const int64_t orr = __shfl_sync(0xffffffffu, orow, rr);
                        const bool lr = __shfl_sync(0xffffffffu, live, rr);
                        const int32_t col = col0 + c + j * (BF16 ? 8 : 4);  // first column of the piece
                        const uint4 x = stg[rr * 8 + (j ^ (rr & 7))];
                        if (lr && col < args.d2) {  // d2 is a multiple of 8: pieces are whole
                            if (BF16)
                                *reinterpret_cast<uint4 *>(static_cast<__nv_bfloat16 *>(args.out) +
                                                           orr * args.d2 + col) = x;
                            else
                                *reinterpret_cast<uint4 *>(static_cast<float *>(args.out) +
                                                           orr * args.d2 + col) = x;
                        }
                    }
                    __syncwarp();
                }
            }
            // this warp is done reading accumulator b
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
        // the warp's TMA stores have completed before the CTA exits
        if (lane == 0) bulk_wait_all();
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == kWarpMma) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(2 * acc_cols));
    }
}

// bT[r][n][k] = b[r][k][n]: the K-major copy of every segment's B block.
template <typename T>
__global__ void k_transpose_b(const T *__restrict__ b, T *__restrict__ bt, int64_t r, int32_t d1,
                              int32_t d2) {
    __shared__ T tile[32][33];
    const int64_t rel = blockIdx.z;
    const int32_t k0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
    const T *src = b + rel * d1 * (int64_t)d2;
    T *dst = bt + rel * d1 * (int64_t)d2;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        int32_t k = k0 + i, n = n0 + threadIdx.x;
        if (k < d1 && n < d2) tile[i][threadIdx.x] = src[(int64_t)k * d2 + n];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        int32_t n = n0 + i, k = k0 + threadIdx.x;
        if (k < d1 && n < d2) dst[(int64_t)n * d1 + k] = tile[threadIdx.x][i];
    }
}

// cuTensorMapEncodeTiled, fetched through the runtime so the library needs no
// link against the driver library.
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

int make_map(CUtensorMap *map, const void *ptr, int bf16, int64_t inner, int64_t outer,
             uint32_t box_inner, uint32_t box_outer) {
    auto fn = encode_fn();
    if (!fn) return fail(BGL_E_CUDA, "cuTensorMapEncodeTiled is not available");
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    cuuint64_t strides[1] = {(cuuint64_t)(inner * (bf16 ? 2 : 4))};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                    2, const_cast<void *>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(BGL_E_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return BGL_OK;
}

size_t smem_bytes(int bn) {
    return 1024 + kStagesA * size_t(kABytes) + kStagesB * size_t(bn) * 128 +
           kEpiWarps * 2 * 32 * kStageRowBytes + 8 * (2 * kStagesA + 2 * kStagesB + 5) + 16;
}

template <bool BF16, bool GATHER>
int launch_tc(dim3 grid, size_t smem, cudaStream_t s, const CUtensorMap &map_a,
              const CUtensorMap &map_b, const CUtensorMap &map_out, const TcArgs &args) {
    BGL_CUDA(cudaFuncSetAttribute(k_gmm_tc<BF16, GATHER>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k_gmm_tc<BF16, GATHER><<<grid, threads_for(GATHER), smem, s>>>(map_a, map_b, map_out, args);
    BGL_LAUNCH_CHECK();
    return BGL_OK;
}

}  // namespace

bool gmm_tensor_core_supported(int64_t d1, int64_t d2, int dtype) {
    if (dtype != BGL_F32 && dtype != BGL_BF16) return false;
    const int64_t elem = dtype == BGL_BF16 ? 2 : 4;
    // TMA rows need 16-byte strides; the epilogue writes 8 columns at a time
    return d1 > 0 && (d1 * elem) % 16 == 0 && d2 > 0 && d2 % 8 == 0 && d1 < (1 << 30) &&
           d2 < (1 << 30);
}

bool gmm_tensor_core_fits(int64_t n, int64_t r, int64_t d2) {
    // TMA coordinates are 32-bit: rows of A and rows of the K-major B copy
    return n < (int64_t(1) << 31) && r * d2 < (int64_t(1) << 31);
}

int gmm_tensor_core(const void *a, const void *b, void *out, const GmmLayout &l, int64_t n,
                    int64_t d1, int64_t r, int64_t d2, int dtype, cudaStream_t s) {
    const bool bf16 = dtype == BGL_BF16;
    const int64_t elem = bf16 ? 2 : 4;
    if (!aligned(a, 16) || !aligned(out, 16) || !l.tc_b)
        return fail(BGL_E_INVALID, "grouped mm: tensor-core path needs 16-byte aligned operands");
    // K-major B
    {
        dim3 grid((unsigned)((d2 + 31) / 32), (unsigned)((d1 + 31) / 32), (unsigned)r);
        if (bf16)
            k_transpose_b<__nv_bfloat16><<<grid, dim3(32, 8), 0, s>>>(
                (const __nv_bfloat16 *)b, (__nv_bfloat16 *)l.tc_b, r, (int32_t)d1, (int32_t)d2);
        else
            k_transpose_b<float><<<grid, dim3(32, 8), 0, s>>>((const float *)b, (float *)l.tc_b, r,
                                                              (int32_t)d1, (int32_t)d2);
        BGL_LAUNCH_CHECK();
    }
    const uint32_t bk = bf16 ? 64 : 32;
    const int64_t kb = (d1 + bk - 1) / bk;
    const int bn = d2 >= 256 ? 256 : (int)((d2 + 15) / 16 * 16);
    const bool gather = l.perm != nullptr;
    CUtensorMap map_a, map_b;
    int rc = make_map(&map_b, l.tc_b, bf16, d1, r * d2, bk, (uint32_t)bn);
    if (rc) return rc;
    CUtensorMap map_out;
    if (gather) {
        // not read: gather_mm's A rows are copied by the kernel's gather warps
        // and its output rows are scattered by the epilogue's own stores
        map_a = map_b;
        map_out = map_b;
        if ((d1 * elem) % 16 != 0)
            return fail(BGL_E_INVALID, "gather_mm: tensor-core rows must be 16-byte multiples");
    } else {
        rc = make_map(&map_a, a, bf16, d1, n, bk, kBM);
        if (rc) return rc;
        // epilogue boxes: 32 rows x 128 bytes (32 fp32 or 64 bf16 columns)
        rc = make_map(&map_out, out, bf16, d2, n, bf16 ? 64 : 32, 32);
        if (rc) return rc;
    }
    TcArgs args;
    args.out = out;
    args.a = a;
    args.a_row_bytes = d1 * elem;
    args.seg_off = l.seg_off;
    args.tile_off = l.tile_off;
    args.perm = l.perm;
    args.r = r;
    args.n = n;
    args.d1 = (int32_t)d1;
    args.d2 = (int32_t)d2;
    args.bn = bn;
    args.kb = (int32_t)kb;
    args.nbn = (int32_t)((d2 + bn - 1) / bn);
    const size_t smem = smem_bytes(bn);
    // persistent: one CTA per SM (its load rings and 2 x BN TMEM columns),
    // never more CTAs than (row tile, column tile) pairs could exist
    int64_t max_work = ((n + kBM - 1) / kBM + r) * args.nbn;
    dim3 grid((unsigned)(max_work < num_sms() ? max_work : num_sms()));
    if (bf16)
        return gather ? launch_tc<true, true>(grid, smem, s, map_a, map_b, map_out, args)
                      : launch_tc<true, false>(grid, smem, s, map_a, map_b, map_out, args);
    return gather ? launch_tc<false, true>(grid, smem, s, map_a, map_b, map_out, args)
                  : launch_tc<false, false>(grid, smem, s, map_a, map_b, map_out, args);
}

}  // namespace bgl

extern "C" int bgl_tc_error(void) {
    int code = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&code, bgl::g_bgl_tc_error, sizeof(int)) != cudaSuccess)
        return bgl::fail(BGL_E_CUDA, "reading the tensor-core error word failed");
    if (code) cudaMemcpyToSymbol(bgl::g_bgl_tc_error, &zero, sizeof(int));
    return code;
}
