// Host/device parameter blocks shared between the C-ABI layer (se12_abi.cu)
// and the kernels. Not part of the public interface (include/se12.h is).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace se12 {

// One SE12 matrix on the device, as the kernels see it.
struct MatrixView {
  const uint8_t* sm;               // [T*4096] tile-major sign|mantissa bytes
  const uint8_t* ec;               // [T*2048] packed 4-bit codes
  const uint8_t* esc;              // [T*16] escape exponent slots
  const uint8_t* bitmap;           // [ceil(T/8)] fallback bitmap, MSB first
  const uint16_t* fallback_raw;    // [F*4096] raw BF16 bits of fallback tiles
  const uint16_t* escape_pos;      // [T*16] derived: tile-flat index of each escape, 0xFFFF unused
  const int32_t* fallback_index;   // [T] derived: rank among fallback tiles, -1 otherwise
  int rows, cols;                  // N, K (unpadded)
  int tile_rows, tile_cols;        // ceil(N/16), ceil(K/256)
  int tiles;                       // tile_rows * tile_cols
  uint8_t codebook[16];            // 15 entries + 1 pad
};

// Arguments of one fused (or dense baseline) GEMV launch: y = x . W^T.
struct GemvArgs {
  MatrixView m;        // for the dense baseline only rows/cols/tile_* are used
  const uint16_t* x;   // [B, ldx] bf16
  int ldx;
  int batch;
  float* y;            // [B, ldy] fp32
  int ldy;
  float* partials;     // [grid][2][16 * 8 * nblocks] stream-K partial rows
  int* counters;       // [tile_rows] arrival counters, zero between calls
  int grid;
  int stages;
};

// Shared-memory carve-up of the GEMV kernels (bytes). The weight area of a
// stage holds either one SE12 tile (sm: 2 x 2048 swizzled halves, ec: 2048
// swizzled) or one raw 16x256 BF16 tile (8192 bytes).
constexpr int kStageWeightBytes = 8192;
constexpr int kXRowStride = 528;        // bytes per batch row of a staged x slice (512 + 16 pad)
constexpr int kLutCopies = 32;          // one LUT column per lane: conflict-free lookups
constexpr int kLutBytes = 256 * kLutCopies * 4;
constexpr int kConsumerWarps = 4;
constexpr int kGemvThreads = (kConsumerWarps + 1) * 32;

inline int x_stage_bytes(int batch) { return (batch * kXRowStride + 127) / 128 * 128; }

inline size_t gemv_smem_bytes(bool raw, int stages, int nblocks, int batch) {
  size_t bytes = 1024;                                      // alignment slack
  bytes += (size_t)stages * kStageWeightBytes;              // weights
  if (!raw) bytes += kLutBytes;                             // pair LUT
  bytes += (size_t)stages * x_stage_bytes(batch);           // x slices
  bytes += (size_t)stages * 64;                             // esc (16) + positions (32) + meta (16)
  bytes += (size_t)kConsumerWarps * 16 * 8 * nblocks * 4;   // row reduction
  bytes += (size_t)stages * 16 + 64;                        // barriers + flags
  return bytes;
}

// Kernel launchers (defined in the .cu files).
cudaError_t launch_gemv(bool raw, const CUtensorMap& map0, const CUtensorMap& map1, const GemvArgs& a, int nblocks,
                        size_t smem, cudaStream_t stream, bool pdl);
cudaError_t launch_prepare(const MatrixView& m, uint16_t* escape_pos, int32_t* fallback_index, cudaStream_t stream);
cudaError_t launch_decode(const MatrixView& m, uint16_t* out, int ldo, cudaStream_t stream);
cudaError_t launch_decode_rows(const MatrixView& m, const int32_t* rows, int nrows, uint16_t* out, int ldo,
                               cudaStream_t stream);
cudaError_t launch_encode_histogram(const uint16_t* w, int rows, int cols, int ldw, uint32_t* counts,
                                    cudaStream_t stream);
cudaError_t launch_encode_tiles(const uint16_t* w, int rows, int cols, int ldw, const uint8_t* codebook,
                                uint8_t* sm, uint8_t* ec, uint8_t* esc, uint8_t* tile_fallback, cudaStream_t stream);
cudaError_t launch_encode_bitmap(const uint8_t* tile_fallback, int tiles, uint8_t* bitmap, int32_t* fallback_index,
                                 int32_t* fallback_count, cudaStream_t stream);
cudaError_t launch_encode_raw(const uint16_t* w, int rows, int cols, int ldw, const int32_t* fallback_index,
                              uint16_t* raw, cudaStream_t stream);
cudaError_t read_device_status(unsigned* out, bool clear);

}  // namespace se12
