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

// Where a lane's V output columns [k0, k0 + V) live in an operand row:
// resolved once per lane (its columns do not change while it walks edges), so
// the broadcast's divide and modulo stay out of the gather loop.
template <int V>
struct ColMap {
    int32_t off;  // operand column of the lane's first output column
    int32_t k0;   // the lane's first output column (for the rare per-element broadcast)
};

template <typename T, int V>
__device__ __forceinline__ ColMap<V> col_map(const Operand<T> &o, int64_t k0) {
    ColMap<V> m;
    m.k0 = (int32_t)k0;
    m.off = o.full ? (int32_t)k0 : (int32_t)((k0 / o.div) % o.width);
    return m;
}

// Loads the lane's V output columns of operand row `row`.
template <typename T, int V>
__device__ __forceinline__ void load_mapped(const Operand<T> &o, int64_t row, const ColMap<V> &m,
                                            T (&r)[V]) {
    const T *base = o.ptr + row * o.width;
    if (o.full) {
        ld_stream(base + m.off, r);
    } else if (o.uniform) {
        T x = __ldg(base + m.off);
#pragma unroll
        for (int i = 0; i < V; ++i) r[i] = x;
    } else {
#pragma unroll
        for (int i = 0; i < V; ++i) r[i] = __ldg(base + ((m.k0 + i) / o.div) % o.width);
    }
}

// Loads output columns [k0, k0 + V) of operand row `row`.
template <typename T, int V>
__device__ __forceinline__ void load_cols(const Operand<T> &o, int64_t row, int64_t k0,
                                          T (&r)[V]) {
    const T *base = o.ptr + row * o.width;
    if (o.full) {
        ld_stream(base + k0, r);
    } else if (o.uniform) {
        T x = __ldg(base + (k0 / o.div) % o.width);
#pragma unroll
        for (int i = 0; i < V; ++i) r[i] = x;
    } else {
#pragma unroll
        for (int i = 0; i < V; ++i) r[i] = __ldg(base + ((k0 + i) / o.div) % o.width);
    }
}

inline bool aligned(const void *p, size_t a) {
    return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

inline int next_pow2(int64_t x) {
    int p = 1;
    while (p < x && p < 32) p <<= 1;
    return p;
}

}  // namespace bgl
