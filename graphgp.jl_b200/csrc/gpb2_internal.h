// gpb2_internal.h -- error plumbing shared by every translation unit of libgraphgp_b200.so.
#pragma once
#include <cstdarg>
#include <cstdint>
#include <cstdio>

#include "../../include/graphgp_b200.h"

namespace gpb2 {

// Thread-local message behind gpb2_last_error(); set_error returns the status it records so a
// failing path can `return set_error(...)`.
int set_error(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
void clear_error();

}  // namespace gpb2

#define GPB2_CUDA_TRY(expr)                                                                   \
    do {                                                                                      \
        cudaError_t _e = (expr);                                                              \
        if (_e != cudaSuccess)                                                                \
            return ::gpb2::set_error(_e == cudaErrorMemoryAllocation ? GPB2_ERR_OOM           \
                                                                     : GPB2_ERR_CUDA,         \
                                     "%s:%d: %s -> %s", __FILE__, __LINE__, #expr,            \
                                     cudaGetErrorString(_e));                                 \
    } while (0)

#define GPB2_TRY(expr)                      \
    do {                                    \
        int _s = (expr);                    \
        if (_s != GPB2_OK) return _s;       \
    } while (0)
