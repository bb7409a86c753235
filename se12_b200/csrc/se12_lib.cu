// Single translation unit of libse12_b200.so: the kernels share the device
// status word g_status, so they are compiled together.
#include "se12_codec.cu"
#include "se12_gemv.cu"
#include "se12_chain.cu"
#include "se12_abi.cu"
