// Single translation unit of liblinearard_b200.so: the generic kernels, the
// sm_100a kernels and the C ABI share the device error word.
#include "lkl_generic.cu"
#include "lkl_sm100.cu"
#include "lkl_api.cu"
#include "lkl_noalloc.cu"
