// SE12 codec kernels for sm_100a: load-time preparation, decode to global
// memory, row decode, and the encoder (packer).
//
// Format (the lws.pack on-disk format, reference src/lws/domain/se12/codec.py):
//   tiles of 16 x 256 weights in row-major tile order; inside a tile the
//   flat index is local_row * 256 + local_col;
//   sm  [T*4096]  (sign << 7) | mantissa of every weight      (codec.py:134)
//   ec  [T*2048]  4-bit code, even flat index in the low nibble (codec.py:310-324)
//   esc [T*16]    exponents of escaped weights in flat order    (codec.py:332-343)
//   fallback_bitmap: tile i -> bit 7 - i%8 of byte i/8          (codec.py:351-353)
//   fallback_raw: int16 bits of every fallback tile, tile order (codec.py:363-365)
// A tile with more than 16 escapes is a fallback tile (codec.py:131-133).
// Padding weights (+0.0) are forced to code 0 (codec.py:120-125).
#include "se12_device.cuh"
#include "se12_internal.h"

namespace se12 {

// ---------------------------------------------------------------- prepare

// One warp per tile: the tile-flat index of every escaped weight, in rank
// order (the order its exponent appears in the tile's esc slots), 0xFFFF in
// unused slots; all 0xFFFF for fallback tiles. This is the information the
// reference recovers per weight with a cumulative count (codec.py:379-391)
// or per (row, k-tile) with a host table (src/lws/adapters/cuda/gemv.py:56-77).
__global__ void prepare_escape_positions(const uint8_t* __restrict__ ec, const uint8_t* __restrict__ bitmap, int tiles,
                                         uint16_t* __restrict__ escape_pos) {
  const int warps_per_block = blockDim.x >> 5;
  const int tile = blockIdx.x * warps_per_block + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (tile >= tiles) return;
  uint16_t* out = escape_pos + static_cast<size_t>(tile) * kEscapeBudget;
  const bool fallback = (bitmap[tile >> 3] >> (7 - (tile & 7))) & 1u;
  if (fallback) {
    if (lane < kEscapeBudget) out[lane] = kNoEscape;
    return;
  }
  // lane covers ec bytes [64*lane, 64*lane + 64) = flat indices [128*lane, 128*lane + 128)
  const uint4* src = reinterpret_cast<const uint4*>(ec + static_cast<size_t>(tile) * (kTileSize / 2) + lane * 64);
  uint32_t words[16];
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    const uint4 u = src[v];
    words[4 * v] = u.x;
    words[4 * v + 1] = u.y;
    words[4 * v + 2] = u.z;
    words[4 * v + 3] = u.w;
  }
  int count = 0;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const uint32_t w = words[k];
    // bit 3 of each nibble of f is set iff that nibble is 0xF
    const uint32_t f = ((w & 0x77777777u) + 0x11111111u) & w & 0x88888888u;
    count += __popc(f);
  }
  int before = count;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int v = __shfl_up_sync(0xFFFFFFFFu, before, d);
    if (lane >= d) before += v;
  }
  const int total = __shfl_sync(0xFFFFFFFFu, before, 31);
  before -= count;  // exclusive
  if (count) {
    int rank = before;
    for (int k = 0; k < 16; ++k) {
      uint32_t f = ((words[k] & 0x77777777u) + 0x11111111u) & words[k] & 0x88888888u;
      while (f) {
        const int bit = __ffs(f) - 1;  // 3, 7, 11, ... : nibble = bit / 4
        f &= f - 1;
        if (rank < kEscapeBudget) out[rank] = static_cast<uint16_t>(lane * 128 + k * 8 + (bit >> 2));
        ++rank;
      }
    }
  }
  if (lane < kEscapeBudget && lane >= total) out[lane] = kNoEscape;
}

// Exclusive scan of the fallback bitmap: rank among fallback tiles, -1 for
// the others (the reference's fallback_offsets, gemv.py:47-53, except that
// non-fallback tiles get -1 instead of a don't-care value).
__global__ void scan_fallback(const uint8_t* __restrict__ bitmap, int tiles, int padded_tiles,
                              int32_t* __restrict__ fallback_index, int32_t* __restrict__ fallback_count) {
  __shared__ int warp_sums[32];
  __shared__ int carry;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < tiles; base += blockDim.x) {
    const int tile = base + tid;
    const int bit = (tile < tiles) ? ((bitmap[tile >> 3] >> (7 - (tile & 7))) & 1) : 0;
    const unsigned m = __ballot_sync(0xFFFFFFFFu, bit);
    const int in_warp = __popc(m & ((1u << lane) - 1u));
    if (lane == 31) warp_sums[warp] = __popc(m);
    __syncthreads();
    if (warp == 0) {
      const int nw = blockDim.x >> 5;
      int v = (lane < nw) ? warp_sums[lane] : 0;
      int incl = v;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int o = __shfl_up_sync(0xFFFFFFFFu, incl, d);
        if (lane >= d) incl += o;
      }
      if (lane < nw) warp_sums[lane] = incl - v;
    }
    __syncthreads();
    const int rank = carry + warp_sums[warp] + in_warp;
    if (tile < tiles) fallback_index[tile] = bit ? rank : -1;
    __syncthreads();
    if (tid == blockDim.x - 1) carry = rank + bit;
    __syncthreads();
  }
  if (tid == 0 && fallback_count) *fallback_count = carry;
  for (int tile = tiles + tid; tile < padded_tiles; tile += blockDim.x) fallback_index[tile] = -1;
}

cudaError_t launch_prepare(const MatrixView& m, uint16_t* escape_pos, int32_t* fallback_index, cudaStream_t stream) {
  if (m.tiles == 0) return cudaSuccess;
  const int warps = 8;
  prepare_escape_positions<<<(m.tiles + warps - 1) / warps, warps * 32, 0, stream>>>(m.ec, m.bitmap, m.tiles, escape_pos);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  // padded to a multiple of 4 tiles: the GEMV copies whole 16-byte groups
  scan_fallback<<<1, 1024, 0, stream>>>(m.bitmap, m.tiles, (m.tiles + 3) & ~3, fallback_index, nullptr);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- decode

// Decodes 32 consecutive weights of one tile row: sm bytes `s0,s1` (2 x 16),
// ec bytes `e` (16). Writes 16 BF16x2 words (low half = lower column).
__device__ __forceinline__ void decode32(uint4 s0, uint4 s1, uint4 e, const uint32_t* lut, uint32_t (&out)[16]) {
  const uint32_t sw[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
  const uint32_t ew[4] = {e.x, e.y, e.z, e.w};
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const uint32_t eword = ew[m >> 1];
    const int b = (m & 1) * 2;
    const uint32_t t0 = lut[(eword >> (8 * b)) & 0xFFu];
    const uint32_t t1 = lut[(eword >> (8 * b + 8)) & 0xFFu];
    out[2 * m] = pair_word(__byte_perm(sw[m], 0, 0x1100), t0);
    out[2 * m + 1] = pair_word(__byte_perm(sw[m], 0, 0x3322), t1);
  }
}

struct DecodeCodebook {
  uint8_t v[16];
};

// Full decode to a row-major [rows, ldo] BF16 matrix (cropped to rows x cols).
// One 256-thread block per pair of tiles; thread -> (tile, local row, 32 columns).
__global__ void __launch_bounds__(256) decode_kernel(const __grid_constant__ MatrixView m, uint16_t* __restrict__ out,
                                                     int ldo) {
  __shared__ uint32_t lut[kMaxSegments][256];  // per segment
  for (int i = threadIdx.x; i < 256 * m.segments; i += blockDim.x) lut[i >> 8][i & 255] = pair_entry(m.codebooks[i >> 8], i & 255);
  __syncthreads();
  const int tile = blockIdx.x * 2 + (threadIdx.x >> 7);
  if (tile >= m.tiles) return;
  const int i = threadIdx.x & 127;
  const int r = i >> 3, c0 = (i & 7) * 32;
  const int tr = tile / m.tile_cols, kt = tile - tr * m.tile_cols;
  const int grow = tr * kTileRows + r;
  if (grow >= m.rows) return;
  const int gcol = kt * kTileCols + c0;
  if (gcol >= m.cols) return;
  uint32_t words[16];
  const int fb = ((m.bitmap[tile >> 3] >> (7 - (tile & 7))) & 1u) ? m.fallback_index[tile] : -1;
  if (fb >= 0) {
    const uint4* src = reinterpret_cast<const uint4*>(m.fallback_raw + static_cast<size_t>(fb) * kTileSize + r * kTileCols + c0);
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const uint4 u = __ldg(src + v);
      words[4 * v] = u.x;
      words[4 * v + 1] = u.y;
      words[4 * v + 2] = u.z;
      words[4 * v + 3] = u.w;
    }
  } else {
    const uint4* smp = reinterpret_cast<const uint4*>(m.sm + static_cast<size_t>(tile) * kTileSize + r * kTileCols + c0);
    const uint4* ecp = reinterpret_cast<const uint4*>(m.ec + static_cast<size_t>(tile) * (kTileSize / 2) + r * 128 + c0 / 2);
    decode32(__ldg(smp), __ldg(smp + 1), __ldg(ecp), lut[segment_of(m, tr)], words);
  }
  uint16_t* dst = out + static_cast<size_t>(grow) * ldo + gcol;
  const int valid = min(32, m.cols - gcol);
  const bool vec = (valid == 32) && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0);
  if (vec) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int v = 0; v < 4; ++v) d4[v] = make_uint4(words[4 * v], words[4 * v + 1], words[4 * v + 2], words[4 * v + 3]);
  } else {
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      if (k < valid) dst[k] = static_cast<uint16_t>(words[k >> 1] >> (16 * (k & 1)));
    }
  }
  if (fb < 0) {
    // escaped weights of this thread's 32 columns (decoded as +0 above)
    const uint16_t* pos = m.escape_pos + static_cast<size_t>(tile) * kEscapeBudget;
    for (int e = 0; e < kEscapeBudget; ++e) {
      const uint32_t p = pos[e];
      if (p == kNoEscape) break;
      const int pr = static_cast<int>(p >> 8), pc = static_cast<int>(p & 255u);
      if (pr == r && pc >= c0 && pc < c0 + 32) {
        const uint32_t smb = m.sm[static_cast<size_t>(tile) * kTileSize + p];
        dst[pc - c0] = static_cast<uint16_t>(bf16_bits(smb, m.esc[static_cast<size_t>(tile) * kEscapeBudget + e]));
      }
    }
  }
}

cudaError_t launch_decode(const MatrixView& m, uint16_t* out, int ldo, cudaStream_t stream) {
  if (m.tiles == 0) return cudaSuccess;
  decode_kernel<<<(m.tiles + 1) / 2, 256, 0, stream>>>(m, out, ldo);
  return cudaGetLastError();
}

// Decodes whole matrix rows in request order: out[i, :] = W[rows[i], :]
// (the reference's WeightDecoder.decode_rows, src/lws/application/ports/gpu/
// weight_decoder.py:26-33, which there decodes the whole tensor first).
// Grid (nrows, tile_cols); 8 threads per 256-column segment, 32 columns each.
__global__ void __launch_bounds__(64) decode_rows_kernel(const __grid_constant__ MatrixView m,
                                                         const int32_t* __restrict__ rows, int nrows,
                                                         uint16_t* __restrict__ out, int ldo) {
  __shared__ uint32_t lut[kMaxSegments][256];  // per segment
  for (int i = threadIdx.x; i < 256 * m.segments; i += blockDim.x) lut[i >> 8][i & 255] = pair_entry(m.codebooks[i >> 8], i & 255);
  __syncthreads();
  const int req = blockIdx.x * 8 + (threadIdx.x >> 3);
  const int kt = blockIdx.y;
  if (req >= nrows) return;
  const int row = rows[req];
  if (row < 0 || row >= m.rows) {
    raise_status(kStatusBadArgument);
    return;
  }
  const int tr = row >> 4, r = row & 15;
  const int tile = tr * m.tile_cols + kt;
  const int c0 = (threadIdx.x & 7) * 32;
  const int gcol = kt * kTileCols + c0;
  if (gcol >= m.cols) return;
  uint32_t words[16];
  const int fb = ((m.bitmap[tile >> 3] >> (7 - (tile & 7))) & 1u) ? m.fallback_index[tile] : -1;
  if (fb >= 0) {
    const uint4* src = reinterpret_cast<const uint4*>(m.fallback_raw + static_cast<size_t>(fb) * kTileSize + r * kTileCols + c0);
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const uint4 u = __ldg(src + v);
      words[4 * v] = u.x;
      words[4 * v + 1] = u.y;
      words[4 * v + 2] = u.z;
      words[4 * v + 3] = u.w;
    }
  } else {
    const uint4* smp = reinterpret_cast<const uint4*>(m.sm + static_cast<size_t>(tile) * kTileSize + r * kTileCols + c0);
    const uint4* ecp = reinterpret_cast<const uint4*>(m.ec + static_cast<size_t>(tile) * (kTileSize / 2) + r * 128 + c0 / 2);
    decode32(__ldg(smp), __ldg(smp + 1), __ldg(ecp), lut[segment_of(m, tr)], words);
  }
  uint16_t* dst = out + static_cast<size_t>(req) * ldo + gcol;
  const int valid = min(32, m.cols - gcol);
#pragma unroll
  for (int k = 0; k < 32; ++k) {
    if (k < valid) dst[k] = static_cast<uint16_t>(words[k >> 1] >> (16 * (k & 1)));
  }
  if (fb < 0) {
    const uint16_t* pos = m.escape_pos + static_cast<size_t>(tile) * kEscapeBudget;
    for (int e = 0; e < kEscapeBudget; ++e) {
      const uint32_t p = pos[e];
      if (p == kNoEscape) break;
      const int pr = static_cast<int>(p >> 8), pc = static_cast<int>(p & 255u);
      if (pr == r && pc >= c0 && pc < c0 + 32) {
        const uint32_t smb = m.sm[static_cast<size_t>(tile) * kTileSize + p];
        dst[pc - c0] = static_cast<uint16_t>(bf16_bits(smb, m.esc[static_cast<size_t>(tile) * kEscapeBudget + e]));
      }
    }
  }
}

cudaError_t launch_decode_rows(const MatrixView& m, const int32_t* rows, int nrows, uint16_t* out, int ldo,
                               cudaStream_t stream) {
  if (nrows == 0 || m.tile_cols == 0) return cudaSuccess;
  dim3 grid((nrows + 7) / 8, m.tile_cols);
  decode_rows_kernel<<<grid, 64, 0, stream>>>(m, rows, nrows, out, ldo);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- encode

// 256-bin histogram of the exponent byte over the real (unpadded) weights
// (the counts the reference's build_codebook sorts, codebook.py:41-59).
__global__ void __launch_bounds__(256) encode_histogram_kernel(const uint16_t* __restrict__ w, int rows, int cols, int ldw,
                                                               uint32_t* __restrict__ counts) {
  __shared__ uint32_t hist[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int vpr = (cols + 7) / 8;  // 8-weight groups per row
  const long long total = static_cast<long long>(rows) * vpr;
  const bool aligned = ((ldw & 7) == 0) && ((reinterpret_cast<uintptr_t>(w) & 15) == 0);
  for (long long v = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; v < total;
       v += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(v / vpr);
    const int c = static_cast<int>(v - static_cast<long long>(row) * vpr) * 8;
    const uint16_t* src = w + static_cast<size_t>(row) * ldw + c;
    if (aligned && c + 8 <= cols) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(src));
      const uint32_t ws[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        atomicAdd(&hist[(ws[k] >> 7) & 0xFFu], 1u);
        atomicAdd(&hist[(ws[k] >> 23) & 0xFFu], 1u);
      }
    } else {
      for (int k = 0; k < 8 && c + k < cols; ++k) atomicAdd(&hist[(src[k] >> 7) & 0xFFu], 1u);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 256; i += blockDim.x)
    if (hist[i]) atomicAdd(&counts[i], hist[i]);
}

cudaError_t launch_encode_histogram(const uint16_t* w, int rows, int cols, int ldw, uint32_t* counts,
                                    cudaStream_t stream) {
  cudaError_t err = cudaMemsetAsync(counts, 0, 256 * sizeof(uint32_t), stream);
  if (err != cudaSuccess) return err;
  if (rows == 0 || cols == 0) return cudaSuccess;
  const long long groups = static_cast<long long>(rows) * ((cols + 7) / 8);
  long long want = (groups + 255) / 256;
  const int blocks = static_cast<int>(want < 148 * 8 ? want : 148 * 8);
  encode_histogram_kernel<<<blocks, 256, 0, stream>>>(w, rows, cols, ldw, counts);
  return cudaGetLastError();
}

struct EncodeCodebook {
  uint8_t v[16];
};

// One 256-thread block per tile. Thread i owns local row i/16 and the 16
// columns (i%16)*16 ..: threads are in tile-flat order, so an exclusive scan
// of per-thread escape counts gives every escape its rank (codec.py:332-343).
__global__ void __launch_bounds__(256) encode_tiles_kernel(const uint16_t* __restrict__ w, int rows, int cols, int ldw,
                                                           int tile_cols, const __grid_constant__ EncodeCodebook book,
                                                           uint8_t* __restrict__ sm, uint8_t* __restrict__ ec,
                                                           uint8_t* __restrict__ esc,
                                                           uint8_t* __restrict__ tile_fallback) {
  __shared__ uint8_t code_of[256];
  __shared__ int warp_counts[8];
  __shared__ uint8_t slots[kEscapeBudget];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < 256) code_of[tid] = kEscapeCode;
  __syncthreads();
  if (tid < kCodebookSize) code_of[book.v[tid]] = static_cast<uint8_t>(tid);
  __syncthreads();
  const int tile = blockIdx.x;
  const int tr = tile / tile_cols, kt = tile - tr * tile_cols;
  const int r = tid >> 4, c0 = (tid & 15) * 16;
  const int grow = tr * kTileRows + r, gcol = kt * kTileCols + c0;
  uint16_t bits[16];
  const uint16_t* src = w + static_cast<size_t>(grow) * ldw + gcol;
  const bool row_ok = grow < rows;
  if (row_ok && gcol + 16 <= cols && ((ldw & 7) == 0) && ((reinterpret_cast<uintptr_t>(src) & 15) == 0)) {
    const uint4 u0 = __ldg(reinterpret_cast<const uint4*>(src));
    const uint4 u1 = __ldg(reinterpret_cast<const uint4*>(src) + 1);
    const uint32_t ws[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      bits[2 * k] = static_cast<uint16_t>(ws[k]);
      bits[2 * k + 1] = static_cast<uint16_t>(ws[k] >> 16);
    }
  } else {
#pragma unroll
    for (int k = 0; k < 16; ++k) bits[k] = (row_ok && gcol + k < cols) ? src[k] : 0;
  }
  uint8_t smb[16], code[16];
  int count = 0;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const uint32_t b = bits[k];
    smb[k] = static_cast<uint8_t>(((b >> 8) & 0x80u) | (b & 0x7Fu));
    const bool valid = row_ok && (gcol + k < cols);
    const uint8_t cd = valid ? code_of[(b >> 7) & 0xFFu] : 0;  // padding -> code 0
    code[k] = cd;
    count += (cd == kEscapeCode);
  }
  // sign|mantissa and packed codes
  uint32_t s4[4], e2[2];
#pragma unroll
  for (int k = 0; k < 4; ++k)
    s4[k] = smb[4 * k] | (smb[4 * k + 1] << 8) | (smb[4 * k + 2] << 16) | (static_cast<uint32_t>(smb[4 * k + 3]) << 24);
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    uint32_t v = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) v |= static_cast<uint32_t>(code[8 * k + j]) << (4 * j);
    e2[k] = v;
  }
  *reinterpret_cast<uint4*>(sm + static_cast<size_t>(tile) * kTileSize + r * kTileCols + c0) = make_uint4(s4[0], s4[1], s4[2], s4[3]);
  *reinterpret_cast<uint2*>(ec + static_cast<size_t>(tile) * (kTileSize / 2) + r * 128 + c0 / 2) = make_uint2(e2[0], e2[1]);

  // rank of this thread's first escape = escapes in earlier threads
  int incl = count;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int o = __shfl_up_sync(0xFFFFFFFFu, incl, d);
    if (lane >= d) incl += o;
  }
  if (lane == 31) warp_counts[warp] = incl;
  if (tid < kEscapeBudget) slots[tid] = 0;
  __syncthreads();
  int before = incl - count, total = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int v = warp_counts[k];
    if (k < warp) before += v;
    total += v;
  }
  const bool fallback = total > kEscapeBudget;
  if (!fallback && count) {
    int rank = before;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      if (code[k] == kEscapeCode) slots[rank++] = static_cast<uint8_t>((bits[k] >> 7) & 0xFFu);
    }
  }
  __syncthreads();
  if (tid < kEscapeBudget) esc[static_cast<size_t>(tile) * kEscapeBudget + tid] = slots[tid];
  if (tid == 0) tile_fallback[tile] = fallback ? 1 : 0;
}

cudaError_t launch_encode_tiles(const uint16_t* w, int rows, int cols, int ldw, const uint8_t* codebook,
                                uint8_t* sm, uint8_t* ec, uint8_t* esc, uint8_t* tile_fallback, cudaStream_t stream) {
  const int tile_rows = (rows + kTileRows - 1) / kTileRows, tile_cols = (cols + kTileCols - 1) / kTileCols;
  const int tiles = tile_rows * tile_cols;
  if (tiles == 0) return cudaSuccess;
  EncodeCodebook book = {};
  for (int i = 0; i < kCodebookSize; ++i) book.v[i] = codebook[i];
  encode_tiles_kernel<<<tiles, 256, 0, stream>>>(w, rows, cols, ldw, tile_cols, book, sm, ec, esc, tile_fallback);
  return cudaGetLastError();
}

// Packs per-tile fallback flags into the bitmap (numpy.packbits order) and
// ranks the fallback tiles.
__global__ void pack_bitmap_kernel(const uint8_t* __restrict__ tile_fallback, int tiles, uint8_t* __restrict__ bitmap) {
  const int byte = blockIdx.x * blockDim.x + threadIdx.x;
  if (byte * 8 >= tiles) return;
  uint32_t v = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int tile = byte * 8 + k;
    if (tile < tiles && tile_fallback[tile]) v |= 1u << (7 - k);
  }
  bitmap[byte] = static_cast<uint8_t>(v);
}

cudaError_t launch_encode_bitmap(const uint8_t* tile_fallback, int tiles, uint8_t* bitmap, int32_t* fallback_index,
                                 int32_t* fallback_count, cudaStream_t stream) {
  if (tiles == 0) return cudaMemsetAsync(fallback_count, 0, sizeof(int32_t), stream);
  const int bytes = (tiles + 7) / 8;
  pack_bitmap_kernel<<<(bytes + 255) / 256, 256, 0, stream>>>(tile_fallback, tiles, bitmap);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  scan_fallback<<<1, 1024, 0, stream>>>(bitmap, tiles, tiles, fallback_index, fallback_count);
  return cudaGetLastError();
}

// Raw bits of every fallback tile, padded with +0.0, in tile-flat order.
__global__ void __launch_bounds__(256) encode_raw_kernel(const uint16_t* __restrict__ w, int rows, int cols, int ldw,
                                                         int tile_cols, const int32_t* __restrict__ fallback_index,
                                                         uint16_t* __restrict__ raw) {
  const int tile = blockIdx.x;
  const int fb = fallback_index[tile];
  if (fb < 0) return;
  const int tr = tile / tile_cols, kt = tile - tr * tile_cols;
  uint16_t* dst = raw + static_cast<size_t>(fb) * kTileSize;
  for (int i = threadIdx.x; i < kTileSize; i += blockDim.x) {
    const int r = i >> 8, c = i & 255;
    const int grow = tr * kTileRows + r, gcol = kt * kTileCols + c;
    dst[i] = (grow < rows && gcol < cols) ? w[static_cast<size_t>(grow) * ldw + gcol] : 0;
  }
}

cudaError_t launch_encode_raw(const uint16_t* w, int rows, int cols, int ldw, const int32_t* fallback_index,
                              uint16_t* raw, cudaStream_t stream) {
  const int tile_rows = (rows + kTileRows - 1) / kTileRows, tile_cols = (cols + kTileCols - 1) / kTileCols;
  const int tiles = tile_rows * tile_cols;
  if (tiles == 0) return cudaSuccess;
  encode_raw_kernel<<<tiles, 256, 0, stream>>>(w, rows, cols, ldw, tile_cols, fallback_index, raw);
  return cudaGetLastError();
}

cudaError_t read_device_status(unsigned* out, bool clear) {
  cudaError_t err = cudaMemcpyFromSymbol(out, g_status, sizeof(unsigned));
  if (err != cudaSuccess) return err;
  if (clear) {
    const unsigned zero = 0;
    err = cudaMemcpyToSymbol(g_status, &zero, sizeof(unsigned));
  }
  return err;
}

cudaError_t set_wait_limit(unsigned long long ns) { return cudaMemcpyToSymbol(g_wait_limit_ns, &ns, sizeof(ns)); }

cudaError_t get_wait_limit(unsigned long long* ns) { return cudaMemcpyFromSymbol(ns, g_wait_limit_ns, sizeof(*ns)); }

}  // namespace se12
