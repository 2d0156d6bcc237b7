// Shared device/host helpers for libbgl: status plumbing, element traits,
// IEEE-exact arithmetic wrappers and vector loads.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cmath>
#include <cstdio>

#include "../../include/bgl.h"

namespace bgl {

// ------------------------------------------------------------ host status
// Records `msg` as this thread's last error and returns `code`.
int fail(int code, const char *fmt, ...);
void clear_error();

#define BGL_CUDA(call)                                                                   \
    do {                                                                                 \
        cudaError_t e_ = (call);                                                         \
        if (e_ != cudaSuccess)                                                           \
            return ::bgl::fail(BGL_E_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

// Checks the launch that was just issued.
#define BGL_LAUNCH_CHECK() BGL_CUDA(cudaGetLastError())

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

int num_sms();  // SMs of the current device (cached per device)

// Tuning parameters settable through bgl_set_param.
struct Params {
    int64_t spmm_min_items = 32;   // merge-path chunk floor (items = rows + edges)
    int64_t spmm_max_chunks = 0;   // cap on chunks, 0 = automatic
    int64_t spmm_split_min = 512;  // rows with at most this many edges are never split
    int64_t softmax_segment_warp = 1;  // segment_softmax: one warp per segment
};
Params &params();

// Carves consecutive 256-byte-aligned regions out of a caller workspace.
struct Carver {
    char *base;
    size_t used = 0;
    explicit Carver(void *p) : base(static_cast<char *>(p)) {}
    template <typename T>
    T *take(size_t count) {
        used = (used + 255) & ~size_t(255);
        T *p = reinterpret_cast<T *>(base ? base + used : nullptr);
        used += count * sizeof(T);
        return p;
    }
};

// ------------------------------------------------------------ device math
// Every arithmetic step goes through an explicitly rounded intrinsic so that
// nvcc cannot contract `acc + x * y` into a fused multiply-add: the
// reference (src/ported.mojo) rounds the message and the accumulation
// separately, and fp64 runs are compared bit for bit.
template <typename T>
struct Arith;

template <>
struct Arith<float> {
    static __device__ __forceinline__ float add(float a, float b) { return __fadd_rn(a, b); }
    static __device__ __forceinline__ float sub(float a, float b) { return __fsub_rn(a, b); }
    static __device__ __forceinline__ float mul(float a, float b) { return __fmul_rn(a, b); }
    static __device__ __forceinline__ float div(float a, float b) { return __fdiv_rn(a, b); }
    static __device__ __forceinline__ float ninf() { return -INFINITY; }
    static __device__ __forceinline__ float pinf() { return INFINITY; }
    static __device__ __forceinline__ float ex(float a) { return expf(a); }
    static __device__ __forceinline__ float fma(float a, float b, float c) { return __fmaf_rn(a, b, c); }
};

template <>
struct Arith<double> {
    static __device__ __forceinline__ double add(double a, double b) { return __dadd_rn(a, b); }
    static __device__ __forceinline__ double sub(double a, double b) { return __dsub_rn(a, b); }
    static __device__ __forceinline__ double mul(double a, double b) { return __dmul_rn(a, b); }
    static __device__ __forceinline__ double div(double a, double b) { return __ddiv_rn(a, b); }
    static __device__ __forceinline__ double ninf() { return -INFINITY; }
    static __device__ __forceinline__ double pinf() { return INFINITY; }
    static __device__ __forceinline__ double ex(double a) { return exp(a); }
    static __device__ __forceinline__ double fma(double a, double b, double c) { return __fma_rn(a, b, c); }
};

// The message functor of src/ported.mojo:92-105.
template <int OP, typename T>
__device__ __forceinline__ T message(T x, T y) {
    if (OP == BGL_OP_ADD) return Arith<T>::add(x, y);
    if (OP == BGL_OP_SUB) return Arith<T>::sub(x, y);
    if (OP == BGL_OP_MUL) return Arith<T>::mul(x, y);
    if (OP == BGL_OP_DIV) return Arith<T>::div(x, y);
    if (OP == BGL_OP_COPY_LHS) return x;
    return y;
}

// ------------------------------------------------------------ vector I/O
template <typename T, int V>
struct VecT;
template <> struct VecT<float, 1> { using type = float; };
template <> struct VecT<float, 2> { using type = float2; };
template <> struct VecT<float, 4> { using type = float4; };
template <> struct VecT<double, 1> { using type = double; };
template <> struct VecT<double, 2> { using type = double2; };

template <typename T, int V>
__device__ __forceinline__ void load_vec(const T *p, T (&r)[V]) {
    using VT = typename VecT<T, V>::type;
    VT v = __ldg(reinterpret_cast<const VT *>(p));
    const T *s = reinterpret_cast<const T *>(&v);
#pragma unroll
    for (int i = 0; i < V; ++i) r[i] = s[i];
}

// Read-only vector load that does not allocate in L1: gathered feature rows
// are touched once per edge and essentially never hit L1.
__device__ __forceinline__ void ld_stream(const float *p, float (&r)[4]) {
    asm("ld.global.nc.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];"
        : "=f"(r[0]), "=f"(r[1]), "=f"(r[2]), "=f"(r[3]) : "l"(p));
}
__device__ __forceinline__ void ld_stream(const float *p, float (&r)[2]) {
    asm("ld.global.nc.L1::no_allocate.v2.f32 {%0, %1}, [%2];" : "=f"(r[0]), "=f"(r[1]) : "l"(p));
}
__device__ __forceinline__ void ld_stream(const float *p, float (&r)[1]) {
    asm("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(r[0]) : "l"(p));
}
__device__ __forceinline__ void ld_stream(const double *p, double (&r)[2]) {
    asm("ld.global.nc.L1::no_allocate.v2.f64 {%0, %1}, [%2];" : "=d"(r[0]), "=d"(r[1]) : "l"(p));
}
__device__ __forceinline__ void ld_stream(const double *p, double (&r)[1]) {
    asm("ld.global.nc.L1::no_allocate.f64 %0, [%1];" : "=d"(r[0]) : "l"(p));
}

template <typename T, int V>
__device__ __forceinline__ void store_vec(T *p, const T (&r)[V]) {
    using VT = typename VecT<T, V>::type;
    VT v;
    T *s = reinterpret_cast<T *>(&v);
#pragma unroll
    for (int i = 0; i < V; ++i) s[i] = r[i];
    *reinterpret_cast<VT *>(p) = v;
}

// Streaming (evict-first) variants for data touched once -- the per-edge
// outputs of gSDDMM and the softmax, the edge-order softmax's logits -- so
// that L2 keeps the small per-node arrays those kernels gather again (CUDA's
// __stcs / __ldcs cache-streaming operators; config 2's u_add_v: 0.57 ->
// 0.51 ms).  Index and edge-id streams stay on the default path (a team reads
// consecutive ids from one line, and L1 serves all but the first), and so do
// the gSpMM and GAT row outputs, which measured no better or slower with it.
template <typename T, int V>
__device__ __forceinline__ void store_stream(T *p, const T (&r)[V]) {
    using VT = typename VecT<T, V>::type;
    VT v;
    T *s = reinterpret_cast<T *>(&v);
#pragma unroll
    for (int i = 0; i < V; ++i) s[i] = r[i];
    __stcs(reinterpret_cast<VT *>(p), v);
}
template <typename T, int V>
__device__ __forceinline__ void load_once(const T *p, T (&r)[V]) {
    using VT = typename VecT<T, V>::type;
    const VT v = __ldcs(reinterpret_cast<const VT *>(p));
    const T *s = reinterpret_cast<const T *>(&v);
#pragma unroll
    for (int i = 0; i < V; ++i) r[i] = s[i];
}

// One operand's view: row stride `width`, output column k reads column
// (k / div) % width.  `full` (width == dout, div == 1) is the fast path.
template <typename T>
struct Operand {
    const T *ptr;
    int64_t width;
    int64_t div;
    bool full;
    bool uniform;  // div % V == 0: one element serves a whole output vector
};

inline bool aligned(const void *p, size_t a) {
    return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

inline int next_pow2(int64_t x) {
    int p = 1;
    while (p < x && p < 32) p <<= 1;
    return p;
}

// ------------------------------------------------------- async row staging
// Per-lane asynchronous copies global -> shared (cp.async, sm_80 and later).
// A lane copies its own V columns of a gathered row into its own shared slot
// and later reads back only what it copied, so the per-thread
// cp.async.wait_group is the only synchronisation: no barrier, no spin.  The
// data in flight holds no registers, so the copy depth is bounded by shared
// memory instead of the register file.
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

// 16-byte copies bypass L1 (.cg), like ld_stream: gathered rows are read once.
template <int BYTES>
__device__ __forceinline__ void cp_async(uint32_t dst, const void *src) {
    static_assert(BYTES == 4 || BYTES == 8 || BYTES == 16, "cp.async copies 4, 8 or 16 bytes");
    if (BYTES == 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], %2;" ::"r"(dst), "l"(src), "n"(BYTES)
                     : "memory");
}
// Reads back a lane's slot: one shared-memory load of V values at a 32-bit
// shared address (volatile, so it stays after the cp.async wait before it).
__device__ __forceinline__ void lds_vec(uint32_t a, float (&r)[4]) {
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(r[0]), "=f"(r[1]), "=f"(r[2]), "=f"(r[3]) : "r"(a));
}
__device__ __forceinline__ void lds_vec(uint32_t a, float (&r)[2]) {
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(r[0]), "=f"(r[1]) : "r"(a));
}
__device__ __forceinline__ void lds_vec(uint32_t a, float (&r)[1]) {
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(r[0]) : "r"(a));
}
__device__ __forceinline__ void lds_vec(uint32_t a, double (&r)[2]) {
    asm volatile("ld.shared.v2.f64 {%0, %1}, [%2];" : "=d"(r[0]), "=d"(r[1]) : "r"(a));
}
__device__ __forceinline__ void lds_vec(uint32_t a, double (&r)[1]) {
    asm volatile("ld.shared.f64 %0, [%1];" : "=d"(r[0]) : "r"(a));
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
// Returns once at most N of this thread's committed groups are still pending.
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// One operand as a lane reads it during a walk: the address of the lane's
// first value in row 0 and the row stride in bytes, so a row's address is one
// 32 x 32 -> 64-bit multiply-add.  `mode` 0: the lane's V values are adjacent
// (a full operand, or any operand read one column at a time); 1: one value
// serves all V columns (uniform broadcast); 2: each of the V values has its
// own broadcast column (a divisor that V does not divide).
template <typename T, int V>
struct LaneCols {
    const char *base;
    uint32_t row_bytes;
    int32_t mode;
    int32_t k0;
};

template <typename T, int V>
__device__ __forceinline__ LaneCols<T, V> lane_cols(const Operand<T> &o, int64_t k0) {
    LaneCols<T, V> c;
    c.row_bytes = (uint32_t)(o.width * (int64_t)sizeof(T));
    c.k0 = (int32_t)k0;
    if (o.full) {
        c.mode = 0;
        c.base = reinterpret_cast<const char *>(o.ptr + k0);
    } else if (o.uniform) {
        c.mode = 1;
        c.base = reinterpret_cast<const char *>(
            o.ptr + ((uint32_t)k0 / (uint32_t)o.div) % (uint32_t)o.width);
    } else {
        c.mode = 2;
        c.base = reinterpret_cast<const char *>(o.ptr);
    }
    return c;
}

// Starts the copy of the lane's values of operand row `row` into shared slot
// `dst` (V * sizeof(T) bytes, aligned to that size).
template <typename T, int V>
__device__ __forceinline__ void stage_row(const LaneCols<T, V> &c, const Operand<T> &o,
                                          int32_t row, uint32_t dst) {
    const char *src = c.base + (uint64_t)(uint32_t)row * c.row_bytes;
    if (c.mode == 0) {
        cp_async<V * sizeof(T)>(dst, src);
    } else if (c.mode == 1) {
        cp_async<sizeof(T)>(dst, src);
    } else {
        const T *r = reinterpret_cast<const T *>(src);
#pragma unroll
        for (int i = 0; i < V; ++i)
            cp_async<sizeof(T)>(dst + i * sizeof(T),
                                r + ((uint32_t)(c.k0 + i) / (uint32_t)o.div) % (uint32_t)o.width);
    }
}

// Loads the lane's values of operand row `row` into registers (the same
// addressing as stage_row, for kernels without a gather ring).
template <typename T, int V>
__device__ __forceinline__ void load_row(const LaneCols<T, V> &c, const Operand<T> &o, int64_t row,
                                         T (&r)[V]) {
    const char *src = c.base + (uint64_t)row * c.row_bytes;
    if (c.mode == 0) {
        ld_stream(reinterpret_cast<const T *>(src), r);
    } else if (c.mode == 1) {
        const T x = __ldg(reinterpret_cast<const T *>(src));
#pragma unroll
        for (int i = 0; i < V; ++i) r[i] = x;
    } else {
        const T *p = reinterpret_cast<const T *>(src);
#pragma unroll
        for (int i = 0; i < V; ++i)
            r[i] = __ldg(p + ((uint32_t)(c.k0 + i) / (uint32_t)o.div) % (uint32_t)o.width);
    }
}

// Reads back what stage_row copied into `slot`.
template <typename T, int V>
__device__ __forceinline__ void read_row(const LaneCols<T, V> &c, const T *slot, T (&r)[V]) {
    if (c.mode == 1) {
        const T x = *slot;
#pragma unroll
        for (int i = 0; i < V; ++i) r[i] = x;
    } else {
        using VT = typename VecT<T, V>::type;
        const VT v = *reinterpret_cast<const VT *>(slot);
        const T *s = reinterpret_cast<const T *>(&v);
#pragma unroll
        for (int i = 0; i < V; ++i) r[i] = s[i];
    }
}

}  // namespace bgl
