// The drop-in kernel module (a cubin a manifest binds by entry name, like the
// reference's source/*.cu modules): the route.cu kernels the entries build on,
// the extern "C" entries of dropin.cu and the grouped GEMMs' entries of
// module_gemm.cu, with no host code.
#include "route.cu"
#include "dropin.cu"
#include "module_gemm.cu"
