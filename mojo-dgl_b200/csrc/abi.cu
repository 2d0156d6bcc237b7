// Status plumbing and process-wide settings of libbgl.
#include <cstdarg>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace bgl {

static thread_local char g_last_error[1024] = "";

int fail(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

void clear_error() { g_last_error[0] = '\0'; }

Params &params() {
    static Params p;
    return p;
}

int num_sms() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (cached[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

}  // namespace bgl

extern "C" {

const char *bgl_last_error(void) { return bgl::g_last_error; }

int bgl_abi_version(void) { return 1; }

int bgl_set_param(const char *name, int64_t value) {
    if (name == nullptr) return bgl::fail(BGL_E_INVALID, "bgl_set_param: null name");
    if (std::strcmp(name, "spmm_min_items") == 0) {
        if (value < 1) return bgl::fail(BGL_E_INVALID, "spmm_min_items must be >= 1");
        bgl::params().spmm_min_items = value;
        return BGL_OK;
    }
    if (std::strcmp(name, "spmm_max_chunks") == 0) {
        if (value < 0) return bgl::fail(BGL_E_INVALID, "spmm_max_chunks must be >= 0");
        bgl::params().spmm_max_chunks = value;
        return BGL_OK;
    }
    if (std::strcmp(name, "spmm_split_min") == 0) {
        if (value < 0) return bgl::fail(BGL_E_INVALID, "spmm_split_min must be >= 0");
        bgl::params().spmm_split_min = value;
        return BGL_OK;
    }
    if (std::strcmp(name, "softmax_segment_warp") == 0) {
        bgl::params().softmax_segment_warp = value != 0;
        return BGL_OK;
    }
    return bgl::fail(BGL_E_INVALID, "bgl_set_param: unknown parameter '%s'", name);
}

}  // extern "C"
