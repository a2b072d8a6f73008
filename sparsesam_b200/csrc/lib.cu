// Single translation unit of libsparsesam_b200.so: the kernels share the device
// error flag and the host caches without relocatable device code.
#include "host_util.cu"
#include "gemm.cu"
#include "perm.cu"
#include "rows.cu"
#include "attention.cu"
#include "capi.cu"
#include "noalloc.cu"
