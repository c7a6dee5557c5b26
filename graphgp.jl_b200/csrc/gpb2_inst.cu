// One kernel set, instantiated for the (T, D, K) given on the command line (-DGPB2_T=float
// -DGPB2_TN=f32 -DGPB2_D=2 -DGPB2_K=8); the Makefile compiles this file once per entry of
// gpb2_kset.h so the heavily unrolled kernels build in parallel.
#include "gpb2_kernels.cuh"

#if !defined(GPB2_T) || !defined(GPB2_TN) || !defined(GPB2_D) || !defined(GPB2_K)
#error "compile with -DGPB2_T, -DGPB2_TN, -DGPB2_D and -DGPB2_K"
#endif

#define GPB2_CAT6(a, b, c, d, e, f) a##b##c##d##e##f
#define GPB2_XCAT6(a, b, c, d, e, f) GPB2_CAT6(a, b, c, d, e, f)

namespace gpb2 {
const Ops<GPB2_T>* GPB2_XCAT6(ops_, GPB2_TN, _d, GPB2_D, _k, GPB2_K)() {
    return Launch<GPB2_T, GPB2_K, GPB2_D>::ops();
}
}  // namespace gpb2
