// gpb2_kset.h -- the (T, D, K) shapes with a compiled kernel set.  gpb2_inst.cu is compiled once
// per entry (see ../Makefile, which carries the same list) and gpb2_registry.cu maps a runtime
// (dtype, D, K) to the entry's Ops table.
#pragma once

#define GPB2_DK(X, T, TN)                                                                     \
    X(T, TN, 2, 4) X(T, TN, 2, 5) X(T, TN, 2, 6) X(T, TN, 2, 8) X(T, TN, 2, 10)               \
    X(T, TN, 2, 12) X(T, TN, 2, 16)                                                           \
    X(T, TN, 3, 4) X(T, TN, 3, 5) X(T, TN, 3, 6) X(T, TN, 3, 8) X(T, TN, 3, 10)               \
    X(T, TN, 3, 12) X(T, TN, 3, 16)                                                           \
    X(T, TN, 1, 4) X(T, TN, 1, 8) X(T, TN, 4, 4) X(T, TN, 4, 8) X(T, TN, 4, 10)

#define GPB2_KSET(X) GPB2_DK(X, float, f32) GPB2_DK(X, double, f64)
