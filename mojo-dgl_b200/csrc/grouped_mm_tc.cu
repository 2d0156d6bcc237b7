// tcgen05 grouped GEMM for segment_mm / gather_mm (replaces the serial
// src/ported.mojo:773-804 and the per-row src/ported.mojo:1089-1130).
//
// One CTA computes a 128-row x BN-column tile of one segment: A rows are
// streamed by TMA in 128-byte K slices (32 fp32 or 64 bf16 values, SWIZZLE_128B),
// B is the segment's (K x N) block pre-transposed to K-major (N rows of K) so
// both operands use the canonical K-major swizzled layout; one elected thread
// issues tcgen05.mma (kind::tf32 for fp32 inputs, kind::f16 with bf16 for
// bf16 inputs) into a 128 x BN fp32 accumulator in tensor memory; the four
// warps then read it back with tcgen05.ld (32 lanes each) and store their rows
// (scattered through `perm` for gather_mm).  Two pipeline stages per CTA and
// two CTAs per SM let one CTA's epilogue overlap the other's loads.
//
// Every mbarrier wait is bounded (kTimeoutNs of %globaltimer); on
// expiry the CTA records an error code in g_bgl_tc_error, stops issuing,
// drains what it issued (again bounded), frees its tensor memory and exits.
#include <cuda.h>
#include <cuda_bf16.h>

#include <mutex>

#include "grouped_mm.cuh"

namespace bgl {

__device__ int g_bgl_tc_error = 0;

namespace {

constexpr int kBM = 128;
constexpr int kStages = 2;
constexpr int kThreads = 128;
constexpr unsigned long long kTimeoutNs = 2000000000ull;  // 2 s per wait

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

// Bounded wait: false (and the error word set) if the phase never completes.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = now_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (now_ns() - t0 > kTimeoutNs) {
            atomicCAS(&g_bgl_tc_error, 0, code);
            return false;
        }
    }
    return true;
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

__device__ __forceinline__ void tmem_ld8(uint32_t addr, uint32_t (&r)[8]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7])
        : "r"(addr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

struct TcArgs {
    void *out;
    const int64_t *seg_off;
    const int64_t *tile_off;
    const int32_t *perm;  // gather_mm: output row of permuted row i
    int64_t r;
    int64_t n;
    int32_t d1;
    int32_t d2;
    int32_t bn;      // N columns of one CTA tile (multiple of 16, <= 256)
    int32_t kb;      // number of 128-byte K slices
};

// Instruction descriptor: fp32 accumulator, A/B format (TF32 = 2, BF16 = 1),
// both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t instr_desc(bool bf16, int n) {
    return (1u << 4) | ((bf16 ? 1u : 2u) << 7) | ((bf16 ? 1u : 2u) << 10) |
           ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

template <bool BF16>
__global__ void __launch_bounds__(kThreads, 2)
    k_gmm_tc(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
             const TcArgs args) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const int64_t tile = blockIdx.x;
    if (tile >= args.tile_off[args.r]) return;
    int64_t lo = 0, hi = args.r;
    while (lo < hi) {
        int64_t mid = (lo + hi + 1) >> 1;
        if (args.tile_off[mid] <= tile) lo = mid; else hi = mid - 1;
    }
    const int64_t rel = lo;
    const int64_t row0 = args.seg_off[rel] + (tile - args.tile_off[rel]) * kBM;
    const int64_t row_end = args.seg_off[rel + 1];
    const int32_t nb = blockIdx.y;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t a_bytes = kBM * 128, b_bytes = (uint32_t)args.bn * 128;
    // stage buffers, each 1024-byte aligned (the SWIZZLE_128B atom)
    uintptr_t base = (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023);
    unsigned char *sa = reinterpret_cast<unsigned char *>(base);
    unsigned char *sb = sa + kStages * a_bytes;
    uint64_t *full = reinterpret_cast<uint64_t *>(sb + kStages * b_bytes);
    uint64_t *empty = full + kStages;
    uint64_t *accum = empty + kStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accum + 1);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    const uint32_t tmem_cols = args.bn <= 32 ? 32 : args.bn <= 64 ? 64 : args.bn <= 128 ? 128 : 256;
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(tmem_cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    const int kb_n = args.kb;

    if (warp == 0 && lane == 0) {
        // TMA producer
        int issued = 0;
        for (int kb = 0; kb < kb_n; ++kb) {
            const int s = kb % kStages;
            if (kb >= kStages && !mbar_wait(&empty[s], ((kb / kStages) - 1) & 1, 1)) break;
            mbar_arrive_expect_tx(&full[s], a_bytes + b_bytes);
            const int32_t kx = kb * (BF16 ? 64 : 32);
            tma_load_2d(sa + s * a_bytes, &map_a, &full[s], kx, (int32_t)row0);
            tma_load_2d(sb + s * b_bytes, &map_b, &full[s], kx,
                        (int32_t)(rel * args.d2 + (int64_t)nb * args.bn));
            issued = kb + 1;
        }
        // drain: every issued stage's loads must have landed before exit
        for (int kb = (issued > kStages ? issued - kStages : 0); kb < issued; ++kb)
            mbar_wait(&full[kb % kStages], (kb / kStages) & 1, 2);
    } else if (warp == 1 && lane == 0) {
        // MMA issuer
        const uint32_t idesc = instr_desc(BF16, args.bn);
        bool ok = true;
        for (int kb = 0; kb < kb_n && ok; ++kb) {
            const int s = kb % kStages;
            ok = mbar_wait(&full[s], (kb / kStages) & 1, 3);
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint64_t ad = smem_desc(smem_u32(sa + s * a_bytes));
            const uint64_t bd = smem_desc(smem_u32(sb + s * b_bytes));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)  // 4 MMAs of 32 bytes of K per 128-byte slice
                mma<BF16>(tmem, ad + kk * 2, bd + kk * 2, idesc, (kb | kk) != 0);
            mma_commit(&empty[s]);
        }
        mma_commit(accum);  // arrives once everything issued above has completed
    }
    __syncwarp();

    // epilogue: all four warps, warp w reads TMEM lanes [32w, 32w + 32)
    const bool ready = mbar_wait(accum, 0, 4);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int64_t row = row0 + warp * 32 + lane;
    const bool live = ready && row < row_end;
    const int64_t orow = live ? (args.perm ? (int64_t)args.perm[row] : row) : 0;
    const int32_t col0 = nb * args.bn;
    for (int c = 0; c < args.bn; c += 8) {
        uint32_t v[8];
        tmem_ld8(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c, v);
        const int32_t col = col0 + c;
        if (!live || col >= args.d2) continue;
        if (BF16) {
            __nv_bfloat16 *o = static_cast<__nv_bfloat16 *>(args.out) + orow * args.d2 + col;
            __align__(16) __nv_bfloat16 h[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) h[i] = __float2bfloat16_rn(__uint_as_float(v[i]));
            *reinterpret_cast<uint4 *>(o) = *reinterpret_cast<const uint4 *>(h);
        } else {
            float *o = static_cast<float *>(args.out) + orow * args.d2 + col;
            reinterpret_cast<float4 *>(o)[0] =
                make_float4(__uint_as_float(v[0]), __uint_as_float(v[1]), __uint_as_float(v[2]),
                            __uint_as_float(v[3]));
            reinterpret_cast<float4 *>(o)[1] =
                make_float4(__uint_as_float(v[4]), __uint_as_float(v[5]), __uint_as_float(v[6]),
                            __uint_as_float(v[7]));
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(tmem_cols));
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

// sorted[i] = a[perm[i]] (gather_mm's rows grouped by relation).
template <typename T>
__global__ void k_gather_rows(const T *__restrict__ a, const int32_t *__restrict__ perm,
                              T *__restrict__ sorted, int64_t n, int32_t d1) {
    const int32_t vec = (d1 * (int32_t)sizeof(T)) % 16 == 0 ? 16 / (int32_t)sizeof(T) : 1;
    const int64_t per_row = d1 / vec;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n * per_row;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = i / per_row, c = (i % per_row) * vec;
        const int64_t src = perm[row];
        if (vec > 1)
            *reinterpret_cast<uint4 *>(sorted + row * d1 + c) =
                *reinterpret_cast<const uint4 *>(a + src * d1 + c);
        else
            sorted[row * d1 + c] = a[src * d1 + c];
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
    return 1024 + kStages * (size_t(kBM) * 128 + size_t(bn) * 128) + 8 * (2 * kStages + 1) + 16;
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

size_t gmm_tc_extra_bytes(int64_t n, int64_t d1, int64_t r, int64_t d2, int dtype, bool gather) {
    const int64_t elem = dtype == BGL_BF16 ? 2 : 4;
    size_t b = size_t(r) * d1 * d2 * elem + 256;            // K-major B
    if (gather) b += size_t(n) * d1 * elem + 256;             // rows grouped by relation
    return b;
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
    const void *a_rows = a;
    if (l.perm) {  // gather_mm: group A's rows by relation first
        int g = (int)((n * (d1 * elem / 16) + 255) / 256);
        if (g > num_sms() * 16) g = num_sms() * 16;
        if (g < 1) g = 1;
        if (bf16)
            k_gather_rows<__nv_bfloat16><<<g, 256, 0, s>>>((const __nv_bfloat16 *)a, l.perm,
                                                           (__nv_bfloat16 *)l.tc_a, n, (int32_t)d1);
        else
            k_gather_rows<float><<<g, 256, 0, s>>>((const float *)a, l.perm, (float *)l.tc_a, n,
                                                   (int32_t)d1);
        BGL_LAUNCH_CHECK();
        a_rows = l.tc_a;
    }
    const int bn = d2 >= 256 ? 256 : (int)((d2 + 15) / 16 * 16);
    const uint32_t bk = bf16 ? 64 : 32;
    CUtensorMap map_a, map_b;
    int rc = make_map(&map_a, a_rows, bf16, d1, n, bk, kBM);
    if (rc) return rc;
    rc = make_map(&map_b, l.tc_b, bf16, d1, r * d2, bk, (uint32_t)bn);
    if (rc) return rc;
    TcArgs args;
    args.out = out;
    args.seg_off = l.seg_off;
    args.tile_off = l.tile_off;
    args.perm = l.perm;
    args.r = r;
    args.n = n;
    args.d1 = (int32_t)d1;
    args.d2 = (int32_t)d2;
    args.bn = bn;
    args.kb = (int32_t)((d1 + bk - 1) / bk);
    const size_t smem = smem_bytes(bn);
    int64_t max_tiles = (n + kBM - 1) / kBM + r;
    dim3 grid((unsigned)max_tiles, (unsigned)((d2 + bn - 1) / bn));
    if (bf16) {
        BGL_CUDA(cudaFuncSetAttribute(k_gmm_tc<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem));
        k_gmm_tc<true><<<grid, kThreads, smem, s>>>(map_a, map_b, args);
    } else {
        BGL_CUDA(cudaFuncSetAttribute(k_gmm_tc<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem));
        k_gmm_tc<false><<<grid, kThreads, smem, s>>>(map_a, map_b, args);
    }
    BGL_LAUNCH_CHECK();
    return BGL_OK;
}

}  // namespace bgl

extern "C" int bgl_tc_error(void) {
    int code = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&code, bgl::g_bgl_tc_error, sizeof(int)) != cudaSuccess)
        return bgl::fail(BGL_E_CUDA, "reading the tensor-core error word failed");
    if (code) cudaMemcpyToSymbol(bgl::g_bgl_tc_error, &zero, sizeof(int));
    return code;
}
