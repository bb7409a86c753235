// Host/device parameter blocks shared between the C-ABI layer (se12_abi.cu)
// and the kernels. Not part of the public interface (include/se12.h is).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace se12 {

// One SE12 matrix on the device, as the kernels see it.
// A matrix may be segmented: the tile-major concatenation of up to
// kMaxSegments matrices with the same columns (for example the q, k and v
// projections of one attention block, which share their input), each with
// its own codebook. Segment s covers tile rows [seg_end[s - 1], seg_end[s]);
// every segment but the last has a multiple of 16 rows. An unsegmented
// matrix is one segment.
constexpr int kMaxSegments = 4;

struct MatrixView {
  const uint8_t* sm;               // [T*4096] tile-major sign|mantissa bytes
  const uint8_t* ec;               // [T*2048] packed 4-bit codes
  const uint8_t* esc;              // [T*16] escape exponent slots
  const uint8_t* bitmap;           // [ceil(T/8)] fallback bitmap, MSB first
  const uint16_t* fallback_raw;    // [F*4096] raw BF16 bits of fallback tiles
  const uint16_t* escape_pos;      // [T*16] derived: tile-flat index of each escape, 0xFFFF unused
  const int32_t* fallback_index;   // [round4(T)] derived: rank among fallback tiles, -1 otherwise
  int rows, cols;                  // N, K (unpadded)
  int tile_rows, tile_cols;        // ceil(N/16), ceil(K/256)
  int tiles;                       // tile_rows * tile_cols
  int segments;                    // 1..kMaxSegments
  int seg_end[kMaxSegments];       // exclusive end tile row of each segment (INT32_MAX past the last)
  uint8_t codebooks[kMaxSegments][16];  // per segment: 15 entries + 1 pad
};

// Segment of tile row tr.
static_assert(kMaxSegments == 4, "segment_of compares against three segment ends");
__host__ __device__ __forceinline__ int segment_of(const MatrixView& m, int tr) {
  return (tr >= m.seg_end[0]) + (tr >= m.seg_end[1]) + (tr >= m.seg_end[2]);
}

// All-reduce of y across the GPUs of a peer group (tensor parallelism with
// the input columns sharded), fused into the GEMV: each finished tile row is
// stored into every rank's receive buffer over peer memory, flagged with the
// call's epoch, and summed in rank order once every rank's row is there.
constexpr int kMaxPeers = 8;

struct PeerArgs {
  int world;                 // 1: no all-reduce
  int rank;
  int rows_cap;              // rows a receive slot holds (>= the matrix rows)
  unsigned long long* recv[kMaxPeers];  // rank s's receive buffer (peer-mapped): [2 parities][world][16 batch][rows_cap]
                                        // words, each epoch << 32 | fp32 bits
  int* epoch;                // this rank's [call counter, CTAs finished]; a call uses counter + 1 (its last CTA bumps it)
  // All-gather mode (gather = 1): this rank's matrix holds rows row0 ..
  // row0 + rows - 1 of a rows_full-row output; the receive buffers are read
  // as [2 parities][16 batch][rows_full] words (rows_full <= world x rows_cap)
  // and y is the whole [B][rows_full] output.
  int gather;
  int row0;
  int rows_full;
};

// Arguments of one fused (or dense baseline) GEMV launch: y = x . W^T.
struct GemvArgs {
  MatrixView m;        // for the dense baseline only rows/cols/tile_* are used
  const uint16_t* x;   // [B, ldx] bf16
  int ldx;
  int batch;
  float* y;            // [B, ldy] fp32
  int ldy;
  float* partials;     // [grid][2][16 rows][16 batch] stream-K partial rows (slot 0 used)
  int* counters;       // [grid] per-CTA "partial published" flags, zero between calls
  int grid;
  int stages;
  int raw_3d;          // dense baseline: 1 = one 3-D box per tile, 0 = four 2-D boxes
  int x_resident;      // 1: all of x in shared memory; 0: x staged per stage
  int row_mode;        // 1: each CTA owns whole tile rows; 0: stream-K over stages
  int full_tiles;      // SE12: 1 = 8-tile stages, a warp per tile; 0 = 4-tile stages, a warp per half tile
  int wide;            // SE12, x resident: 1 = one CTA per SM, kWideGroups groups of 4 warps taking 4-tile stages in turn
  PeerArgs peers;      // world == 1: plain GEMV
};

// Pipeline geometry of the GEMV kernels. One stage holds consecutive tiles
// of the linear tile sequence, either
//   4 tiles, consumer warp w taking half w % 2 (128 columns) of tile w / 2, or
//   8 tiles, consumer warp w taking tile w, its two halves in turn (SE12
//   only: half the per-stage overhead per weight, twice the staged x), or
//   4 tiles in the wide layout (SE12 with x resident, one CTA per SM):
//   kWideGroups groups of 4 consumer warps take the stages in turn (group
//   c the stages i with i % kWideGroups == c), warp w taking tile w % 4.
//   18 warps (16 consumers) leave 96 registers a thread. (5 groups, 22
//   warps, leave 80 and spill more: batch 4 and 8 steps 2-3 % slower.)
// SE12 weights arrive as 3-D TMA boxes [64 rows][2 halves][128 B] of sm
// (16 KB) and 2-D boxes [64 rows][128 B] of ec (8 KB), both with the 128-byte
// swizzle: one of each per 4 tiles, the ec boxes after the stage's sm boxes.
// The dense baseline takes one 3-D box [16 rows][4 x 64 columns] (8 KB) per
// tile. x is either resident (all of x[B, K] in shared memory, one bulk copy
// per batch row per CTA) or, when that does not fit, staged per stage by the
// producer warp's lanes with cp.async.
constexpr int kSe12BoxTiles = 4;
__host__ __device__ constexpr int stage_tiles(bool full_tiles) { return full_tiles ? 8 : 4; }
__host__ __device__ constexpr int stage_weight_bytes(bool raw, bool full_tiles) {
  return stage_tiles(full_tiles) * (raw ? 8192 : 6144);
}
constexpr int kXRowStride = 576;        // bytes per (tile, batch row) x slice when staged: 512 + 64 pad
// A GEMV CTA: its consumer warps (8, or 20 in the wide layout), then the
// producer warp (TMA / bulk copies), then the reducer warp (sums the
// consumers' row partials).
constexpr int kConsumerWarps = 8;
constexpr int kWideGroups = 4;
// Kernel builds (the GEMV kernel's LAYOUT): classic (up to two CTAs per SM),
// wide, and solo (the classic layout where shared memory holds one CTA per
// SM, built for one CTA per SM).
constexpr int kLayoutClassic = 0;
constexpr int kLayoutWide = 1;
constexpr int kLayoutSolo = 2;
__host__ __device__ constexpr int consumer_warps(bool wide) { return wide ? kWideGroups * 4 : kConsumerWarps; }
__host__ __device__ constexpr int gemv_threads(bool wide) { return (consumer_warps(wide) + 2) * 32; }
// Escape records (escape positions, escape slots, fallback indices) of
// kRecGroupTiles consecutive tiles (two SE12 stages) are copied into shared
// memory together, into one of kRecSlots slots: [16 tiles][16] u16
// positions, [16][16] u8 slots, [16 + 4] i32 fallback indices.
constexpr int kRecGroupTiles = 16;
constexpr int kRecSlots = 3;
// The wide layout keeps more stages in flight (its record groups are 4
// stages, up to 3 of them live at once, plus the one issued ahead).
__host__ __device__ constexpr int rec_slots(bool wide) { return wide ? 4 : kRecSlots; }
constexpr int kRecPosOffset = 0;
constexpr int kRecEscOffset = kRecGroupTiles * 32;
constexpr int kRecFbOffset = kRecEscOffset + kRecGroupTiles * 16;
constexpr int kRecFbTiles = kRecGroupTiles + 4;  // copied from the 4-tile-aligned tile at or before the group
constexpr int kRecSlotBytes = kRecFbOffset + kRecFbTiles * 4;
constexpr size_t kCoResidentSmem = 112 * 1024;  // two CTAs fit on one SM
constexpr size_t kMaxSmemPerCta = 227 * 1024;   // one CTA per SM (sm_100 opt-in maximum)

// Bytes per batch row of resident x: K rounded up to whole tiles (256
// columns; the columns past K hold zeros), plus 64 so consecutive rows start
// in different bank groups.
__host__ __device__ inline int x_resident_stride(int cols) { return (cols + 255) / 256 * 512 + 64; }

inline size_t x_stage_bytes(bool full_tiles, int batch) {
  return ((size_t)stage_tiles(full_tiles) * batch * kXRowStride + 127) / 128 * 128;
}

// (wide: the wide layout, whose stages are 4 tiles: full_tiles must be false)
inline size_t gemv_smem_bytes(bool raw, bool full_tiles, bool x_resident, int stages, int batch, int cols,
                              bool wide = false) {
  size_t per_stage = stage_weight_bytes(raw, full_tiles) + (x_resident ? 0 : x_stage_bytes(full_tiles, batch));
  size_t bytes = 1024;                                                  // alignment slack
  bytes += (size_t)stages * per_stage;
  if (x_resident) bytes += (size_t)batch * x_resident_stride(cols);
  bytes += 2 * (size_t)consumer_warps(wide) * 16 * batch * 4;          // two row-reduction buffers
  if (!raw) bytes += (size_t)rec_slots(wide) * kRecSlotBytes;           // escape records
  bytes += (size_t)stages * 16 + 128;                                   // barriers
  return bytes;
}

// ------------------------------------------------------------------ chains
// A chain is a sequence of GEMVs run by one persistent launch (se12_chain.cu):
// op j reads its x only once every CTA has finished op j - 1.
constexpr int kChainSlots = 2;            // TMA slots per consumer warp
constexpr int kChainMaxWarps = 15;        // consumer warps per CTA (+ the control warp: 4 warps per SM sub-partition, 128 registers)
constexpr uint32_t kChainSlotSe12 = 6144; // sm (4096 B) + ec (2048 B) of one tile
constexpr uint32_t kChainSlotRaw = 8192;  // one dense BF16 tile
constexpr int kChainMaxOps = 4096;

// One op of a chain, in device memory (the TMA descriptors must be 64-byte
// aligned and stay unchanged while a launch runs).
struct alignas(64) ChainOp {
  CUtensorMap sm_map;            // SE12: sm [16T rows][2][128 B], box one tile; dense: W, box one tile
  CUtensorMap ec_map;            // SE12: ec [16T rows][128 B], box one tile
  const uint32_t* records;       // SE12: [T][16] tile records (se12_matrix_prepare_records)
  const uint16_t* fallback_raw;  // SE12: [F][4096] raw bits of fallback tiles
  const uint16_t* x;             // [batch][ldx] bf16
  float* y;                      // [batch][ldy] fp32
  int ldx, ldy;
  int rows, cols;                // the matrix
  int tile_cols;                 // its tile columns
  int k0, k1;                    // tile-column range this op multiplies (a column split of the matrix)
  int tiles;                     // tile rows x (k1 - k0)
  int x_cols;                    // columns of x this op reads: min(cols, 256 k1) - 256 k0
  int accumulate;                // 1: y += result (an earlier op wrote the other columns' sum)
  int ar_index;                  // >= 0: rows all-reduced over the peer group (the chain's ar_index-th such op)
  int raw_3d;                    // dense: one 3-D box per tile (cols % 64 == 0) or four 2-D boxes
  int segments;
  int seg_end[kMaxSegments];     // exclusive end tile row per segment (INT32_MAX past the last)
  alignas(16) uint32_t tab[kMaxSegments][4]; // decode table per segment (table_byte of codes 0..15, four per word); read as uint4
};
static_assert(offsetof(ChainOp, tab) % 16 == 0, "the kernel loads a segment's table with one 16-byte load");

struct ChainParams {
  const ChainOp* ops;
  const int* starts;    // [n_ops][grid + 1]: op j's tiles [starts[c], starts[c + 1]) belong to CTA c
  int n_ops;
  int batch;
  int consumers;        // consumer warps per CTA (the CTA has one more: the control warp)
  int x_stride;         // bytes per batch row of x in shared memory (= 64 mod 128)
  int x_bytes;          // bytes of the x buffer
  int n_ar;             // ops with an all-reduce
  unsigned* done;       // [n_ops] CTAs that finished op j, over all launches
  unsigned* gen;        // [2]: launches completed, CTAs that left the current launch
  float* partials;      // [grid][2][16 * 16] a CTA's sums of the rows it shares with other CTAs
  unsigned* rowcnt;     // [n_ops][grid][2] tiles summed of a row shared by CTAs (zero between launches)
  PeerArgs peers;
};

size_t chain_smem_bytes(bool raw, int consumers, int x_bytes, int batch);
cudaError_t set_wait_limit(unsigned long long ns);
cudaError_t get_wait_limit(unsigned long long* ns);

// Kernel launchers (defined in the .cu files).
cudaError_t launch_chain(bool raw, const ChainParams& p, int grid, size_t smem, cudaStream_t stream);
cudaError_t launch_prepare_records(const MatrixView& m, uint32_t* records, cudaStream_t stream);
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
