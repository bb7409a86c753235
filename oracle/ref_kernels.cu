// Launchers for the reference's own CUDA kernels, compiled UNCHANGED from
// the reference source tree for sm_100a by oracle/build_ref.py (the
// reference compiles them with NVRTC at run time; nvcc takes the same
// source ahead of time). Test and comparison infrastructure only: the
// parity tests run these kernels against the oracle, and bench.py's
// reference arm times them beside the reference's CPU path. Nothing of the
// product links or calls this library.
//
// Kernels (src/lws/adapters/cuda/kernels/):
//   lws_gemv_se12      gemv_se12.cu:50-142   one warp per (output row, batch)
//   lws_gemv_raw_bf16  gemv_raw_bf16.cu:18-56
// Their launch shape is the reference's default heuristic
// (src/lws/domain/launch/heuristic.py:46-51), computed by the caller.
#include <cuda_runtime.h>

#include "gemv_se12.cu"
#include "gemv_raw_bf16.cu"

extern "C" int ref_gemv_se12(const unsigned char* sm, const unsigned char* ec, const unsigned char* esc,
                             const unsigned char* codebook, const unsigned char* fallback_bitmap,
                             const int* fallback_offsets, const short* fallback_raw, const int* row_escape_offset,
                             const float* x, float* y, int n, int k, int b, int blocks, int threads, void* stream) {
  lws_gemv_se12<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      sm, ec, esc, codebook, fallback_bitmap, fallback_offsets, fallback_raw, row_escape_offset, x, y, n, k, b);
  return static_cast<int>(cudaGetLastError());
}

extern "C" int ref_gemv_raw_bf16(const unsigned short* w, const float* x, float* y, int n, int k, int b, int blocks,
                                 int threads, void* stream) {
  lws_gemv_raw_bf16<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(w, x, y, n, k, b);
  return static_cast<int>(cudaGetLastError());
}
