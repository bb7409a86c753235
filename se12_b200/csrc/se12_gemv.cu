// Fused SE12 decode + GEMV for sm_100a:  y[B, N] = x[B, K] . W[N, K]^T
//
// Replaces the reference's lws_gemv_se12 (src/lws/adapters/cuda/kernels/
// gemv_se12.cu:50-142), which runs one warp per (row, batch) with byte loads
// and re-reads the weights once per batch element. Design here:
//
// * Stream-K over the tile sequence. The matrix is the linear sequence of
//   its T tiles in memory order (tile-row major, 16x256 weights each), cut
//   into stages of 8 consecutive tiles. CTA c (two per SM) owns either whole
//   tile rows (row mode) or a contiguous run of stages (stream-K). Tile rows
//   entirely inside a CTA's run are written directly; a tile row split
//   between CTAs is finished by the CTA holding its first tile, which adds
//   the later CTAs' published partials in CTA order (deterministic, no
//   floating-point atomics).
// * Warp-specialised pipeline. A producer warp moves each stage's sm bytes
//   with one 3-D TMA load ([128 rows][2 halves][128 B]) and its ec bytes
//   with one 2-D TMA load ([128 rows][128 B]), both 128-byte swizzled, onto
//   one mbarrier per stage; the escape records of 16 tiles at a time come
//   with three bulk copies. Eight consumer warps: warp w takes tile w of
//   every stage, its two 128-column halves in turn. A reducer warp sums the
//   consumers' per-row partials, so consumers never wait for each other.
// * Decode in registers straight into mma.sync fragments, with no table in
//   memory: the 16-entry code -> exponent table lives in four registers and
//   is indexed with byte permutes (prmt), 8 codes at a time. Escaped weights
//   enter the MMA with exponent 0 (|w| < 2^-126) and their exact w * x is
//   added in fp32 afterwards from the per-tile escape position list.
//   Fallback tiles are read raw.
// * bf16 m16n8k16 tensor-core MMA with fp32 accumulation; batch padded to
//   multiples of 8. A thread's operands are rows g and g + 8 and four groups
//   of 8 consecutive columns (32k + 8t, k = 0..3, of its half); the MMA k
//   order is permuted per thread the same way for x. Every shared-memory
//   read is bank-conflict free.
// * Two CTAs per SM (shared memory under half an SM, 96 registers a
//   thread): the second CTA's warps hide the first one's latencies.
// * Programmatic dependent launch: the kernel lets the next kernel in the
//   stream launch at once; its CTAs start as SMs free up, prefetch their
//   first stages of weights, and wait (griddepcontrol.wait) only before
//   reading x and writing y.
//
// The dense BF16 baseline (RAW = true) runs the same pipeline over a plain
// row-major BF16 matrix (the reference's lws_gemv_raw_bf16,
// src/lws/adapters/cuda/kernels/gemv_raw_bf16.cu:18-56).
#include "se12_device.cuh"
#include "se12_internal.h"

namespace se12 {

__device__ __forceinline__ int unit_start(int c, int units, int grid) {
  return static_cast<int>((static_cast<long long>(units) * c) / grid);
}

// First tile of CTA c's run (stream-K, stages of `stage` tiles).
__device__ __forceinline__ int tile_start(int c, int units, int grid, int tiles, int stage) {
  return min(unit_start(c, units, grid) * stage, tiles);
}

// CTA whose run contains tile i.
__device__ __forceinline__ int tile_owner(int i, int units, int grid, int stage) {
  const long long u = i / stage;
  return static_cast<int>(((u + 1) * grid - 1) / units);
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t selector) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(selector));
  return d;
}

// (a & m) | (b & ~m)
__device__ __forceinline__ uint32_t select_bits(uint32_t a, uint32_t b, uint32_t m) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xE4;" : "=r"(d) : "r"(a), "r"(b), "r"(m));
  return d;
}

// Exponent byte of code c as the decode table stores it: rotated right by
// one bit, so that its top bit is the exponent's lowest bit (bit 7 of the
// BF16, in its low byte) and its low 7 bits the exponent's upper bits (bits
// 8..14, in its high byte). The escape code maps to exponent 0.
__host__ __device__ __forceinline__ uint32_t table_byte(const uint8_t* codebook, int c) {
  const uint32_t e = (c == kEscapeCode) ? 0u : codebook[c];
  return ((e >> 1) | (e << 7)) & 0xFFu;
}

// Decodes 8 consecutive weights of one row (sign|mantissa bytes in s, codes
// in the nibbles of e, weight i in bits 4i..4i+3) into four BF16x2 words
// p[0..3] = columns (0,1), (2,3), (4,5), (6,7). tab[0..3] hold table_byte
// for codes 0..15 (code c in byte c % 4 of tab[c / 4]).
//  * prmt selects bytes by 3-bit selectors: codes mod 8 look up tab[0..1]
//    and tab[2..3] in two permutes per 4 codes, and a byte mask built from
//    each code's bit 3 (a selector nibble with bit 3 set copies a byte's
//    top bit) picks between them.
//  * A BF16's low byte is the mantissa bits (0x7F) of its sm byte and the
//    top bit of its table byte (the exponent's lowest bit); its high byte
//    is the sm byte's sign bit and the table byte's other 7 bits. Two
//    selects build the four low and the four high bytes of 4 weights at
//    once, two permutes interleave them: 4 instructions per 4 weights.
__device__ __forceinline__ void decode8(uint2 s, uint32_t e, const uint32_t (&tab)[4], uint32_t (&p)[4]) {
  const uint32_t sel03 = e & 0x77777777u;   // selectors for weights 0..3 (low 16 bits)
  const uint32_t sel47 = __umulhi(sel03, 0x10000u);  // weights 4..7: sel03 >> 16 on the multiply pipe (the shift pipe is the busier one)
  const uint32_t e4 = e << 4;                // bit 3 of the even codes at a byte's top bit
  const uint32_t hi03 = prmt(e4, e, 0xD9C8u);  // 0xFF where code >= 8: bytes of e4/e for weights 0,1,2,3
  const uint32_t hi47 = prmt(e4, e, 0xFBEAu);  // weights 4..7
  const uint32_t x03 = select_bits(prmt(tab[2], tab[3], sel03), prmt(tab[0], tab[1], sel03), hi03);
  const uint32_t x47 = select_bits(prmt(tab[2], tab[3], sel47), prmt(tab[0], tab[1], sel47), hi47);
  const uint32_t lo03 = select_bits(s.x, x03, 0x7F7F7F7Fu);  // low bytes of weights 0..3
  const uint32_t up03 = select_bits(s.x, x03, 0x80808080u);  // high bytes
  const uint32_t lo47 = select_bits(s.y, x47, 0x7F7F7F7Fu);
  const uint32_t up47 = select_bits(s.y, x47, 0x80808080u);
  p[0] = prmt(lo03, up03, 0x5140u);  // [lo0, up0, lo1, up1]
  p[1] = prmt(lo03, up03, 0x7362u);  // [lo2, up2, lo3, up3]
  p[2] = prmt(lo47, up47, 0x5140u);
  p[3] = prmt(lo47, up47, 0x7362u);
}

// Padding weights (columns >= K of the last tile column) are +0.0 in the
// packed tile with code 0, so they decode to +2^(codebook[0] - 127); against
// the zeros that x holds there they contribute exactly 0, unless
// codebook[0] == 255 (an infinite padding weight). For that case this
// rewrites, in shared memory, the codes of this thread's padding weights to
// the escape code, which decodes to +0. Each thread patches only the ec
// words it reads itself. Out of line: only such matrices call it.
__device__ __noinline__ void force_padding_escapes(uint8_t* sm8, uint32_t e_addr, uint32_t e_xor, int col0, int valid) {
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t* word = reinterpret_cast<uint32_t*>(sm8 + e_addr + r * 1024 + ((16u * k) ^ e_xor));
      uint32_t v = *word;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (col0 + 32 * k + i >= valid) v |= 0xFu << (4 * i);
      *word = v;
    }
}

template <typename T>
__device__ __forceinline__ T lds_at(const uint8_t* smem, uint32_t offset) {
  return *reinterpret_cast<const T*>(smem + offset);
}

// Two-level accumulation: the MMAs of one half-tile (128 columns) sum into
// fresh accumulators, which are then added to the running sums with plain
// fp32 adds. A tensor-core accumulator carried across a whole tile row adds
// every product into an ever larger partial sum; with large weights (the
// escape-stress points: 1 % of the weights x1024) and long rows that lost
// up to 2e-3 of the output against fp64, where summing per half-tile keeps
// the error at the level of a plain fp32 dot product.
template <int NB>
__device__ __forceinline__ void zero_acc(float (&a)[2][NB][4]) {
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) a[h][nb][0] = a[h][nb][1] = a[h][nb][2] = a[h][nb][3] = 0.f;
}

template <int NB>
__device__ __forceinline__ void add_acc(float (&acc)[2][NB][4], const float (&part)[2][NB][4]) {
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[h][nb][q] += part[h][nb][q];
}

// LAYOUT: kLayoutClassic (two CTAs per SM: 96 registers a thread),
// kLayoutWide, or kLayoutSolo (the classic layout in a configuration whose
// shared memory holds one CTA per SM: compiled for one CTA per SM, so the
// two-block accumulators of batch 9..16 need not spill).
template <int NB, bool RAW, bool XRES, bool FULL, bool AR, int LAYOUT>
__global__ void __launch_bounds__(gemv_threads(LAYOUT == kLayoutWide), LAYOUT == kLayoutClassic ? 2 : 1)
    gemv_kernel(const __grid_constant__ CUtensorMap map0, const __grid_constant__ CUtensorMap map1, const GemvArgs a) {
  constexpr bool WIDE = LAYOUT == kLayoutWide;
  static_assert(!(RAW && FULL), "the dense baseline runs 4-tile stages");
  static_assert(!WIDE || (!RAW && XRES && !FULL && !AR), "the wide layout is SE12 with x resident");
  constexpr int kWeightBytes = stage_weight_bytes(RAW, FULL);
  constexpr int kStage = stage_tiles(FULL);             // tiles per stage
  constexpr int kRecStages = kRecGroupTiles / kStage;   // stages per escape-record slot
  constexpr bool kTilePerWarp = FULL || WIDE;           // a consumer warp multiplies whole tiles
  constexpr int kCons = consumer_warps(WIDE);           // consumer warps
  constexpr int kStageWarps = WIDE ? kStage : kConsumerWarps;  // consumer warps that take each stage
  constexpr int kProducer = kCons;                      // TMA / bulk copies
  constexpr int kReducer = kCons + 1;                   // sums the consumers' row partials
  constexpr int kRS = rec_slots(WIDE);                  // escape-record slots
  static_assert(!WIDE || kWideGroups >= kRecStages, "a wide-layout warp takes at most one stage of a record group");
  extern __shared__ __align__(1024) uint8_t smem_dynamic[];
  // All dynamic shared memory is addressed as smem_dynamic + 32-bit offset,
  // so every access compiles to a shared-memory instruction with 32-bit
  // address arithmetic. `pad` aligns the weight buffers to 1024 bytes (the
  // 128-byte TMA swizzle needs it).
  const uint32_t pad = (1024u - (smem_addr(smem_dynamic) & 1023u)) & 1023u;
  uint8_t* const sm8 = smem_dynamic;

  // Kernel arguments, read once into registers.
  const int S = a.stages;
  const int B = a.batch;
  const int KT = a.m.tile_cols;
  const int T = a.m.tiles;
  const int K = a.m.cols;
  const int N = a.m.rows;
  const int G = a.grid;
  const int ldx = a.ldx, ldy = a.ldy;
  const uint16_t* const xg = a.x;
  float* const yg = a.y;
  float* const partials = a.partials;
  int* const counters = a.counters;
  const uint8_t* const esc_g = a.m.esc;
  const uint16_t* const pos_g = a.m.escape_pos;
  const int32_t* const fbindex_g = a.m.fallback_index;
  const uint16_t* const fbraw_g = a.m.fallback_raw;
  const int raw_3d = a.raw_3d;
  const int kpad8 = (K + 7) & ~7;

  // ------------------------------------------------------------ shared memory (offsets into sm8)
  const uint32_t xrs = static_cast<uint32_t>(x_resident_stride(K));                    // resident x: bytes per batch row
  const uint32_t xstage = (kStage * B * kXRowStride + 127) / 128 * 128;           // staged x: bytes per stage
  const uint32_t o_w = pad;                                                            // S x weights
  const uint32_t o_x = o_w + S * kWeightBytes;                                         // x (resident or staged)
  const uint32_t o_red = o_x + (XRES ? B * xrs : S * xstage);                          // [2][8][16][B] floats
  const uint32_t o_rec = o_red + 2 * kCons * 16 * B * 4;                               // escape record slots
  const uint32_t o_bar = o_rec + (RAW ? 0 : kRS * kRecSlotBytes);
  uint64_t* const full = reinterpret_cast<uint64_t*>(sm8 + o_bar);  // [S] stage loaded
  uint64_t* const empty = full + S;                                 // [S] stage consumed
  uint64_t* const xbar = empty + S;                                 // resident x loaded
  uint64_t* const xready = xbar + 1;                                // resident x loaded and its tail zeroed
  uint64_t* const deposited = xready + 1;                           // [2] all warps' row partials written
  uint64_t* const redfree = deposited + 2;                          // [2] row partials summed
  uint64_t* const rec_full = redfree + 2;                           // [kRS] records loaded
  uint64_t* const rec_empty = rec_full + kRS;                       // [kRS] records consumed
  float* const red = reinterpret_cast<float*>(sm8 + o_red);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int units = (T + kStage - 1) / kStage;
  // This CTA's run of tiles [tstart, tend): whole tile rows (row mode) or
  // a run of stages (stream-K); its stages start at tstart.
  int tstart, tend;
  if (a.row_mode) {
    const long long tile_rows = a.m.tile_rows;
    tstart = static_cast<int>(tile_rows * blockIdx.x / G) * KT;
    tend = static_cast<int>(tile_rows * (blockIdx.x + 1) / G) * KT;
  } else {
    tstart = tile_start(blockIdx.x, units, G, T, kStage);
    tend = tile_start(blockIdx.x + 1, units, G, T, kStage);
  }
  const int nstages = (tend - tstart + kStage - 1) / kStage;
  const int tr_first = tstart / KT;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      // resident x: the weights' expect_tx arrival; staged x: + the "x issued" arrival
      mbar_init(&full[s], XRES ? 1 : 2);
      mbar_init(&empty[s], kStageWarps);
    }
    mbar_init(xbar, 1);
    mbar_init(xready, 1);
    for (int p = 0; p < 2; ++p) {
      mbar_init(&deposited[p], kCons);
      mbar_init(&redfree[p], 1);
    }
    for (int r = 0; r < kRS; ++r) {
      mbar_init(&rec_full[r], 1);
      mbar_init(&rec_empty[r], kCons);
    }
    fence_barrier_init();
  }
  // decode table of each segment: table_byte of codes 0..15, four per word
  __shared__ uint4 seg_tab[kMaxSegments];
  if (!RAW && tid < a.m.segments) {
    uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int c = 0; c < 16; ++c) w[c >> 2] |= table_byte(a.m.codebooks[tid], c) << (8 * (c & 3));
    seg_tab[tid] = make_uint4(w[0], w[1], w[2], w[3]);
  }
  if (XRES) {
    // columns kpad8 .. 256 KT - 1 of every resident x row are zero
    const int tail = KT * kTileCols - kpad8;  // a multiple of 8 columns
    for (int i = tid; i < B * (tail / 8); i += blockDim.x) {
      const int b = i / (tail / 8), c = kpad8 + 8 * (i - b * (tail / 8));
      *reinterpret_cast<uint4*>(sm8 + o_x + b * xrs + 2 * c) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  __syncthreads();
  grid_launch_dependents();

  if (warp == kProducer) {
    // ------------------------------------------------------------ producer
    const uint64_t pol_w = policy_evict_first();
    const uint64_t pol_x = policy_evict_last();
    if (lane == 0) {
      prefetch_tmap(&map0);
      if (!RAW) prefetch_tmap(&map1);
    }
    const int prologue = min(nstages, S);
    // the weights of stage i: 2 TMA loads (SE12) or one per tile (dense)
    auto issue_weights = [&map0, &map1, sm8, o_w, full, tend, KT, tstart, lane, pol_w, raw_3d](int i, int s) {
      if (lane == 0) {
        const int tile0 = tstart + i * kStage;
        const int ntl = min(kStage, tend - tile0);
        uint8_t* w = sm8 + o_w + s * kWeightBytes;
        if (RAW) {
          mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(ntl) * 8192u);
          int tr = tile0 / KT, kt = tile0 - tr * KT;
          for (int j = 0; j < ntl; ++j) {
            if (raw_3d) {
              tma_load_3d(w + j * 8192, &map0, 0, kt * 4, tr * kTileRows, &full[s], pol_w);
            } else {
#pragma unroll
              for (int c = 0; c < 4; ++c)
                tma_load_2d(w + j * 8192 + c * 2048, &map0, kt * kTileCols + c * 64, tr * kTileRows, &full[s], pol_w);
            }
            if (++kt == KT) {
              kt = 0;
              ++tr;
            }
          }
        } else {
          // one sm and one ec box per 4 tiles; boxes past the matrix's
          // last tile read zeros and still count their full bytes
          mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(kWeightBytes));
#pragma unroll
          for (int q = 0; q < kStage / kSe12BoxTiles; ++q) {
            const int row = (tile0 + q * kSe12BoxTiles) * kTileRows;
            tma_load_3d(w + q * (kSe12BoxTiles * 4096), &map0, 0, 0, row, &full[s], pol_w);
            tma_load_2d(w + kStage * 4096 + q * (kSe12BoxTiles * 2048), &map1, 0, row, &full[s], pol_w);
          }
        }
      }
      __syncwarp();
    };
    // staged x of stage i. A tile column whose 256 columns all lie inside K:
    // one 512-byte bulk copy per (tile, batch row) slice, the slices spread
    // over the lanes (x rows start 16-byte aligned: ldx % 8 == 0). The
    // ragged last tile column: lane l copies 16-byte chunk l (columns 8 l ..
    // 8 l + 7) of each slice with cp.async, columns past K written as zeros
    // (the chunk holding column K with a plain load and a mask).
    auto issue_x = [sm8, o_x, full, xg, ldx, xstage, tend, KT, K, B, tstart, lane, pol_x](int i, int s) {
      const int tile0 = tstart + i * kStage;
      const int ntl = min(kStage, tend - tile0);
      const int kt0 = tile0 % KT;
      int whole = 0;  // tiles of the stage whose columns all lie inside K
      bool ragged = false;
      for (int j = 0, kt = kt0; j < ntl; ++j) {
        if ((kt + 1) * kTileCols <= K) ++whole;
        else ragged = true;
        if (++kt == KT) kt = 0;
      }
      if (lane == 0 && whole) mbar_expect_tx(&full[s], static_cast<uint32_t>(whole * B) * 512u);
      __syncwarp();
      for (int q = lane; q < ntl * B; q += 32) {
        const int j = q / B, b = q - j * B;
        int kt = kt0 + j;
        if (kt >= KT) kt -= KT;
        if ((kt + 1) * kTileCols <= K)
          bulk_load(sm8 + o_x + s * xstage + (j * B + b) * kXRowStride,
                    xg + static_cast<size_t>(b) * ldx + kt * kTileCols, 512u, &full[s], pol_x);
      }
      int kt = kt0;
      for (int j = 0; ragged && j < ntl; ++j) {
        const int col = kt * kTileCols + lane * 8;
        if (++kt == KT) kt = 0;
        if (col - lane * 8 + kTileCols <= K) continue;  // a whole tile: copied above
        for (int b = 0; b < B; ++b) {
          uint8_t* dst = sm8 + o_x + s * xstage + (j * B + b) * kXRowStride + lane * 16;
          const uint16_t* src = xg + static_cast<size_t>(b) * ldx + col;
          if (col + 8 <= K) {
            cp_async_16_ca(dst, src);
          } else {
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (col < K) {
              v = *reinterpret_cast<const uint4*>(src);
              uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                if (col + 2 * q >= K) w[q] = 0u;
                else if (col + 2 * q + 1 >= K) w[q] &= 0xFFFFu;
              }
            }
            *reinterpret_cast<uint4*>(dst) = v;
          }
        }
      }
      if (ragged) cp_async_mbar_arrive(&full[s]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[s]);
      __syncwarp();
    };
    // Escape records of record group r (tiles 16 r .. 16 r + 15 of this
    // CTA's run): three bulk copies into slot r % kRS. Positions (32 B per
    // tile) and slots (16 B per tile) start 16-byte aligned at any tile; the
    // fallback indices (4 B per tile) are copied from the 4-tile-aligned tile
    // at or before the group (the table is padded to a multiple of 4 tiles).
    auto issue_records = [sm8, o_rec, rec_full, rec_empty, pos_g, esc_g, fbindex_g, tend, tstart, nstages, lane,
                          pol_w](int r) -> bool {
      if (RAW || r * kRecStages >= nstages) return true;
      bool good = true;
      if (lane == 0) {
        const int slot = r % kRS;
        if (r >= kRS) good = mbar_wait_sleep(&rec_empty[slot], static_cast<uint32_t>(r / kRS - 1) & 1u);
        if (good) {
          const int t0 = tstart + r * kRecGroupTiles;
          const int n = min(kRecGroupTiles, tend - t0);
          const int t0a = t0 & ~3;
          const int n4 = (t0 - t0a + n + 3) & ~3;
          uint8_t* dst = sm8 + o_rec + slot * kRecSlotBytes;
          mbar_arrive_expect_tx(&rec_full[slot], static_cast<uint32_t>(n * 48 + n4 * 4));
          bulk_load(dst + kRecPosOffset, pos_g + static_cast<size_t>(t0) * kEscapeBudget, n * 32, &rec_full[slot], pol_w);
          bulk_load(dst + kRecEscOffset, esc_g + static_cast<size_t>(t0) * kEscapeBudget, n * 16, &rec_full[slot], pol_w);
          bulk_load(dst + kRecFbOffset, fbindex_g + t0a, n4 * 4, &rec_full[slot], pol_w);
        }
      }
      return __shfl_sync(0xFFFFFFFFu, good ? 1 : 0, 0) != 0;
    };
    // Records run one group ahead of the weights: before stage i is issued,
    // every group up to i / kRecStages + 1. Group g reuses the slot of group
    // g - 3, released when the consumers finish its last stage, which lies
    // before stage i - kRecStages (already issued); the prologue's groups
    // (at most 0..2) find their slots free.
    int next_group = 0;
    auto records_upto = [&issue_records, &next_group](int i) -> bool {
      for (const int want = i / kRecStages + 1; next_group <= want; ++next_group)
        if (!issue_records(next_group)) return false;
      return true;
    };
    for (int i = 0; i < prologue; ++i) {
      records_upto(i);
      issue_weights(i, i);
    }
    grid_dependency_wait();  // x is produced by the previous kernel in the stream
    if (XRES) {
      const uint32_t xbytes = static_cast<uint32_t>(kpad8) * 2u;
      if (lane == 0) mbar_arrive_expect_tx(xbar, xbytes * static_cast<uint32_t>(B));
      __syncwarp();
      if (lane < B) bulk_load(sm8 + o_x + lane * xrs, xg + static_cast<size_t>(lane) * ldx, xbytes, xbar, pol_x);
      __syncwarp();
      if (K & 7) {
        // the copy brought columns K .. kpad8 - 1 as the caller left them:
        // zero them, then release x to the consumers
        const bool landed = mbar_wait(xbar, 0);
        if (landed && lane < B)
          for (int c = K; c < kpad8; ++c) *reinterpret_cast<uint16_t*>(sm8 + o_x + lane * xrs + 2 * c) = 0;
        __syncwarp();
        if (lane == 0) mbar_arrive(xready);
      }
    } else {
      for (int i = 0; i < prologue; ++i) issue_x(i, i);
    }
    // stage i goes to slot s = i % S; its empty barrier completes phase
    // i / S - 1 when the consumers release the slot's previous stage
    int s = 0;
    uint32_t ph = 1u;
    for (int i = prologue; i < nstages; ++i) {
      if (!records_upto(i)) break;
      if (!mbar_wait_sleep(&empty[s], ph ^ 1u)) break;
      issue_weights(i, s);
      if (!XRES) issue_x(i, s);
      if (++s == S) {
        s = 0;
        ph ^= 1u;
      }
    }
    return;
  }

  if (warp == kReducer) {
    // ------------------------------------------------------------ reducer
    // Tile rows tr_first .. tr_last end in this CTA, in order. For each: wait
    // for the eight consumer warps' partials and sum them in warp order.
    //  * A row entirely in this CTA: write it to y.
    //  * A row that started in an earlier CTA (only this CTA's first row):
    //    publish the sum (partials slot 0) with a release flag.
    //  * A row that started here and continues into later CTAs (only this
    //    CTA's last row, which it reaches last): acquire the later CTAs'
    //    flags -- they processed the row first, at the start of their runs
    //    -- add their partials in CTA order, write y and clear the flags.
    // Deterministic (CTA order), no atomics. Every CTA of the grid is
    // resident or done before a dependent grid may launch, so the flag
    // waits cannot be starved; they are bounded all the same.
    // Peer all-reduce: this call's epoch is the rank's call counter + 1; the
    // last CTA to finish (every CTA counts itself once, after reading the
    // counter) bumps it, so that every CTA of a call reads the same value.
    const PeerArgs& P = a.peers;
    auto finish_call = [&]() {
      if (AR && lane == 0) {
        __threadfence();
        if (atomicAdd(P.epoch + 1, 1) == G - 1) {
          atomicExch(P.epoch + 1, 0);
          atomicAdd(P.epoch, 1);
        }
      }
    };
    // All-gather mode: once this CTA's rows are out, it waits for its slice
    // of the whole output (every rank's rows, this rank's included) and
    // writes it to y as plain fp32. Slices are even cuts of the B x rows_full
    // words over the grid, so every CTA -- one without rows included -- takes
    // part, and a rank's call ends only when its whole output is there.
    auto unpack_gather = [&](int ep) {
      const size_t gbase = static_cast<size_t>(ep & 1) * 16 * P.rows_full;
      const unsigned long long* mine = P.recv[P.rank] + gbase;
      const long long total = static_cast<long long>(B) * P.rows_full;
      const long long i0 = total * blockIdx.x / G, i1 = total * (blockIdx.x + 1) / G;
      bool arrived = true;
      for (long long i = i0 + lane; i < i1; i += 32) {
        const int b = static_cast<int>(i / P.rows_full), row = static_cast<int>(i - static_cast<long long>(b) * P.rows_full);
        const unsigned long long* src = mine + static_cast<size_t>(b) * P.rows_full + row;
        const unsigned long long w = ld_word_sys(src);
        unsigned bits = static_cast<unsigned>(w);
        bool got = static_cast<unsigned>(w >> 32) == static_cast<unsigned>(ep);
        if (!got) got = wait_word_sys(src, static_cast<unsigned>(ep), &bits);
        arrived = arrived && got;
        if (got) yg[static_cast<size_t>(b) * ldy + row] = __uint_as_float(bits);
      }
      __syncwarp();
      (void)arrived;  // a word that never came left its element unwritten and raised the status word
    };
    if (tend <= tstart) {
      if (AR) {
        grid_dependency_wait();
        if (P.gather) unpack_gather(__ldcg(P.epoch) + 1);
        finish_call();
      }
      return;
    }
    const int tr_last = (tend - 1) / KT;
    const int outs = 16 * B;  // <= 256: up to 8 values per lane
    grid_dependency_wait();   // y and the workspace may be in use by the previous kernel
    const int epoch = AR ? __ldcg(P.epoch) + 1 : 0;
    for (int tr = tr_first; tr <= tr_last; ++tr) {
      const int lr = tr - tr_first, pb = lr & 1;
      if (!mbar_wait(&deposited[pb], static_cast<uint32_t>(lr >> 1) & 1u)) break;
      const float* buf = red + pb * kCons * 16 * B;
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int idx = lane + 32 * j;
        v[j] = 0.f;
        if (idx < outs) {
#pragma unroll
          for (int ww = 0; ww < kCons; ++ww) v[j] += buf[ww * 16 * B + idx];
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&redfree[pb]);
      const bool starts = tr * KT >= tstart;
      const bool ends = (tr + 1) * KT <= tend;
      if (!starts) {
        // contributor: publish this CTA's partial of the row
        float* part = partials + static_cast<size_t>(blockIdx.x) * 2 * (16 * 16);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int idx = lane + 32 * j;
          if (idx < outs) {
            const int row = idx / B, b = idx - row * B;
            part[b * 16 + row] = v[j];
          }
        }
        __syncwarp();
        if (lane == 0) st_release_gpu(&counters[blockIdx.x], 1);
        continue;
      }
      bool good = true;
      int c_hi = blockIdx.x;
      if (!ends) {
        // finisher: add the later contributors' partials, in CTA order
        c_hi = tile_owner((tr + 1) * KT - 1, units, G, kStage);
        for (int c = blockIdx.x + 1 + lane; c <= c_hi; c += 32) good = wait_flag_gpu(&counters[c]) && good;
        good = __all_sync(0xFFFFFFFFu, good);
        __syncwarp();
        for (int c = blockIdx.x + 1; c <= c_hi; ++c) {
          const float* part = partials + static_cast<size_t>(c) * 2 * (16 * 16);
          float p[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int idx = lane + 32 * j;
            const int row = idx / B, b = idx - row * B;
            p[j] = (idx < outs) ? __ldcg(part + b * 16 + row) : 0.f;
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) v[j] += p[j];
        }
      }
      if (AR && good && P.gather) {
        // All-gather: each value of the row, with this call's epoch in the
        // same 64-bit word, into every rank's receive buffer at the row's
        // place in the whole output (this rank's own included); every CTA
        // unpacks its slice of the whole output once its rows are out.
        const size_t gbase = static_cast<size_t>(epoch & 1) * 16 * P.rows_full;
        const unsigned long long tag = static_cast<unsigned long long>(static_cast<unsigned>(epoch)) << 32;
        for (int r = 0; r < P.world; ++r) {
          unsigned long long* dst = P.recv[r] + gbase;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int idx = lane + 32 * j;
            const int row = idx / B, b = idx - row * B;
            const int grow = tr * kTileRows + row;
            if (idx < outs && grow < N)
              st_word_sys(dst + static_cast<size_t>(b) * P.rows_full + P.row0 + grow, tag | __float_as_uint(v[j]));
          }
        }
      } else if (AR && good) {
        // All-reduce of the row across the peer group: store each value,
        // with this call's epoch in the same 64-bit word, into every rank's
        // receive slot (this rank's own included) for this epoch's parity;
        // then wait until every rank's words for the row carry the epoch and
        // sum them in rank order, so that every rank writes the same bits.
        // A word is stored whole, so the data is its own flag (no fence).
        // A rank can be at most one call ahead of another (it needs the
        // other's rows of the call in between), so two parities keep a slot
        // from being overwritten while it is read.
        const size_t slot = static_cast<size_t>(16) * P.rows_cap;
        const size_t base = static_cast<size_t>((epoch & 1) * P.world) * slot;
        const unsigned long long tag = static_cast<unsigned long long>(static_cast<unsigned>(epoch)) << 32;
        for (int r = 0; r < P.world; ++r) {
          unsigned long long* dst = P.recv[r] + base + P.rank * slot;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int idx = lane + 32 * j;
            const int row = idx / B, b = idx - row * B;
            const int grow = tr * kTileRows + row;
            if (idx < outs && grow < N)
              st_word_sys(dst + static_cast<size_t>(b) * P.rows_cap + grow, tag | __float_as_uint(v[j]));
          }
        }
        const unsigned long long* mine = P.recv[P.rank] + base;
        bool arrived = true;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int idx = lane + 32 * j;
          const int row = idx / B, b = idx - row * B;
          const int grow = tr * kTileRows + row;
          if (idx < outs && grow < N) {
            const unsigned long long* src = mine + static_cast<size_t>(b) * P.rows_cap + grow;
            // every rank's word in flight at once; poll again only those
            // that have not arrived
            unsigned long long w[kMaxPeers];
#pragma unroll
            for (int r = 0; r < kMaxPeers; ++r)
              if (r < P.world) w[r] = ld_word_sys(src + r * slot);
            float sum = 0.f;
#pragma unroll
            for (int r = 0; r < kMaxPeers; ++r) {
              if (r < P.world) {
                unsigned bits = static_cast<unsigned>(w[r]);
                if (static_cast<unsigned>(w[r] >> 32) != static_cast<unsigned>(epoch))
                  arrived = wait_word_sys(src + r * slot, static_cast<unsigned>(epoch), &bits) && arrived;
                sum += __uint_as_float(bits);
              }
            }
            v[j] = sum;
          }
        }
        good = __all_sync(0xFFFFFFFFu, arrived);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int idx = lane + 32 * j;
        if (idx < outs) {
          const int row = idx / B, b = idx - row * B;
          const int grow = tr * kTileRows + row;
          if (grow < N && good && !(AR && P.gather)) yg[static_cast<size_t>(b) * ldy + grow] = v[j];
        }
      }
      for (int c = blockIdx.x + 1 + lane; c <= c_hi; c += 32) counters[c] = 0;
    }
    __syncwarp();
    if (AR && P.gather) unpack_gather(epoch);
    finish_call();
    return;
  }

  // -------------------------------------------------------------- consumers
  // 8-tile stages (FULL): warp w decodes tile w of every stage, its two
  // 128-column halves in turn. 4-tile stages: warp w takes half w % 2 of
  // tile w / 2. Wide layout: warp w decodes tile w % 4 of the stages of its
  // group w / 4, both halves in turn.
  const int jw = FULL ? warp : (WIDE ? (warp & 3) : (warp >> 1));  // tile of the stage this warp multiplies
  const int hw = kTilePerWarp ? 0 : (warp & 1);                     // its (first) half
  const int g = lane >> 2, t = lane & 3;
  // decode table of the current tile's segment (seg_tab[cur_seg]), loaded
  // when a tile of another segment comes up
  uint32_t tab[4] = {0u, 0u, 0u, 0u};
  int cur_seg = -1;
  // an infinite padding weight needs its code rewritten (force_padding_escapes):
  // codebook[0] of the segment is 255, whose table byte is 0xFF
  bool pad_inf = false;

  // Per-thread shared-memory offsets (stage 0, tile jw, half hw), fixed for
  // the kernel. Thread (g, t) owns rows g, g + 8 of its tile and, in a half,
  // the column groups 32 k + 8 t .. + 7 for k = 0..3. Row g + 8 lies a
  // constant distance after row g; the group offset is a compile-time value
  // XOR a per-thread swizzle term, so four registers hold the layout (with
  // whole tiles, half 1 lies a lane-dependent distance after half 0, recomputed
  // where it is used).
  uint32_t w_base, w_xor, e_base, e_xor;
  if (RAW) {
    // [16 rows][4 x 64-col chunks][128 B] per tile (3-D box; swizzle phase (4 row + chunk) & 7)
    // or [4 chunks][16 rows][128 B] (2-D boxes; swizzle phase row & 7)
    w_base = jw * 8192 + (raw_3d ? (4 * g + 2 * hw) * 128 : (2 * hw) * 2048 + g * 128);
    w_xor = raw_3d ? static_cast<uint32_t>((4 * g + 2 * hw) & 7) : static_cast<uint32_t>(g);
    e_base = e_xor = 0;
  } else {
    // sm: [16 kStage rows][2 halves][128 B], swizzle phase (2 row + half)
    // & 7; 16-byte block 2 k + t / 2 of the half.
    // ec: [16 kStage rows][128 B] after the sm boxes, swizzle phase row & 7;
    // 16-byte block 4 half + k.
    const uint32_t R0 = 16 * jw + g;
    const uint32_t X = (2 * R0 + hw) & 7;  // same for row R0 + 8
    w_base = (2 * R0 + hw) * 128 + ((((t >> 1) ^ X) & 1) << 4) + 8 * (t & 1);
    w_xor = (X & 6) << 4;                   // group k: + ((32 k) ^ w_xor)
    e_base = kStage * 4096 + R0 * 128 + (((4 * hw) ^ (R0 & 4)) << 4) + 4 * t;
    e_xor = (R0 & 3) << 4;                  // group k: + ((16 k) ^ e_xor)
  }
  // x of batch row g + 8 nb at column 128 hw + 8 t (+ 32 k, + 128 for half
  // 1 with whole tiles) of a tile
  const uint32_t x_thread = XRES ? o_x + static_cast<uint32_t>(g) * xrs + (128 * hw + 8 * t) * 2
                                 : o_x + (jw * B + g) * kXRowStride + (128 * hw + 8 * t) * 2;
  const uint32_t x_nb_step = XRES ? 8 * xrs : 8 * kXRowStride;

  bool ok = true;

  // two independent accumulator sets (column groups 0, 2 and 1, 3)
  float acc[2][NB][4];
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) acc[h][nb][0] = acc[h][nb][1] = acc[h][nb][2] = acc[h][nb][3] = 0.f;

  // This warp's A fragments (rows g and g + 8, its 128 columns) of its
  // current tile: [group k][pair].
  uint32_t frag0[4][4], frag1[4][4];

  // Fills frag0 / frag1 with half hw + h of this warp's tile of stage s (h =
  // 1 only with whole tiles): decoded SE12 weights, the raw bits of a fallback tile
  // (fbi >= 0), or dense BF16 weights. Needs no x, so it may run before the
  // dependency wait.
  auto load_frags = [&](int s, int kt, int fbi, int h) {
    const uint32_t wst = o_w + s * kWeightBytes;
    if (RAW) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        // chunk m = 2 hw + k / 2, 16-byte column block sc = 4 (k % 2) + t
        const uint32_t m1 = k >> 1, sc = 4 * (k & 1) + t;
        uint32_t off0, off1;
        if (raw_3d) {
          off0 = w_base + m1 * 128 + ((sc ^ ((w_xor + m1) & 7)) << 4);
          off1 = off0 + 32 * 128;  // row + 8: same swizzle phase
        } else {
          off0 = w_base + m1 * 2048 + ((sc ^ w_xor) << 4);
          off1 = off0 + 8 * 128;
        }
        const uint4 v0 = lds_at<uint4>(sm8, wst + off0);
        const uint4 v1 = lds_at<uint4>(sm8, wst + off1);
        frag0[k][0] = v0.x; frag0[k][1] = v0.y; frag0[k][2] = v0.z; frag0[k][3] = v0.w;
        frag1[k][0] = v1.x; frag1[k][1] = v1.y; frag1[k][2] = v1.z; frag1[k][3] = v1.w;
      }
      return;
    }
    if (__builtin_expect(fbi >= 0, 0)) {
      // fallback tile: its raw BF16 bits from global memory
      const uint16_t* raw = fbraw_g + static_cast<size_t>(fbi) * kTileSize + 128 * (hw + h) + 8 * t;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint4 v0 = __ldg(reinterpret_cast<const uint4*>(raw + g * kTileCols + 32 * k));
        const uint4 v1 = __ldg(reinterpret_cast<const uint4*>(raw + (g + 8) * kTileCols + 32 * k));
        frag0[k][0] = v0.x; frag0[k][1] = v0.y; frag0[k][2] = v0.z; frag0[k][3] = v0.w;
        frag1[k][0] = v1.x; frag1[k][1] = v1.y; frag1[k][2] = v1.z; frag1[k][3] = v1.w;
      }
      return;
    }
    // half 1 (hw = 0): sm 16-byte block 2 k + t / 2 -> (2 k + t / 2) ^ 1 on
    // the next 128-byte line (whose swizzle phase is odd); ec block k -> 4 +
    // k, 64 bytes later or (row bit 2 set in the swizzle) earlier
    const uint32_t wb = wst + w_base + (h ? 144u - ((static_cast<uint32_t>(lane) & 2u) << 4) : 0u);
    const uint32_t eb = wst + e_base + (h ? 64u - ((static_cast<uint32_t>(lane) & 16u) << 3) : 0u);
    if (__builtin_expect(pad_inf, 0) && kt == KT - 1)
      force_padding_escapes(sm8, eb, e_xor, 128 * (hw + h) + 8 * t, K - kt * kTileCols);
    {
      uint2 sv0[4], sv1[4];
      uint32_t ev0[4], ev1[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t wo = wb + ((32u * k) ^ w_xor);
        const uint32_t eo = eb + ((16u * k) ^ e_xor);
        sv0[k] = lds_at<uint2>(sm8, wo);
        sv1[k] = lds_at<uint2>(sm8, wo + 16 * 128);   // row + 8: 16 half-rows of 128 B later
        ev0[k] = lds_at<uint32_t>(sm8, eo);
        ev1[k] = lds_at<uint32_t>(sm8, eo + 8 * 128);
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        decode8(sv0[k], ev0[k], tab, frag0[k]);
        decode8(sv1[k], ev1[k], tab, frag1[k]);
      }
    }
  };

  // Multiplies the fragments (half hw + h) with x (tile column kt of stage
  // s) into acc.
  auto mma_tile = [&](int s, int kt, int h) {
    const uint32_t xt = (XRES ? x_thread + kt * (kTileCols * 2) : x_thread + s * xstage) + 256 * h;
    float part[2][NB][4];
    zero_acc(part);
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      const bool have = nb * 8 + g < B;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint4 xv = make_uint4(0, 0, 0, 0);
        if (have) xv = lds_at<uint4>(sm8, xt + nb * x_nb_step + 64 * k);
        mma_bf16_16816(part[k & 1][nb], frag0[k][0], frag1[k][0], frag0[k][1], frag1[k][1], xv.x, xv.y);
        mma_bf16_16816(part[k & 1][nb], frag0[k][2], frag1[k][2], frag0[k][3], frag1[k][3], xv.z, xv.w);
      }
    }
    add_acc(acc, part);
  };

  // Decodes half hw + h of this warp's tile of stage s and multiplies it
  // with x one 32-column group at a time, so that only one group's
  // fragments are live (8 registers) and the compiler can overlap a group's
  // decode with the previous group's MMAs. SE12 tiles that are neither
  // fallback tiles nor hold infinite padding weights.
  auto decode_mma = [&](int s, int kt, int h) {
    const uint32_t wst = o_w + s * kWeightBytes;
    const uint32_t wb = wst + w_base + (h ? 144u - ((static_cast<uint32_t>(lane) & 2u) << 4) : 0u);
    const uint32_t eb = wst + e_base + (h ? 64u - ((static_cast<uint32_t>(lane) & 16u) << 3) : 0u);
    const uint32_t xt = (XRES ? x_thread + kt * (kTileCols * 2) : x_thread + s * xstage) + 256 * h;
    float part[2][NB][4];
    zero_acc(part);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t wo = wb + ((32u * k) ^ w_xor);
      const uint32_t eo = eb + ((16u * k) ^ e_xor);
      uint32_t f0[4], f1[4];
      decode8(lds_at<uint2>(sm8, wo), lds_at<uint32_t>(sm8, eo), tab, f0);
      decode8(lds_at<uint2>(sm8, wo + 16 * 128), lds_at<uint32_t>(sm8, eo + 8 * 128), tab, f1);
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        uint4 xv = make_uint4(0, 0, 0, 0);
        if (nb * 8 + g < B) xv = lds_at<uint4>(sm8, xt + nb * x_nb_step + 64 * k);
        mma_bf16_16816(part[k & 1][nb], f0[0], f1[0], f0[1], f1[1], xv.x, xv.y);
        mma_bf16_16816(part[k & 1][nb], f0[2], f1[2], f0[3], f1[3], xv.z, xv.w);
      }
    }
    add_acc(acc, part);
  };

  // Adds the exact products of the warp's escaped weights: in the MMA they
  // decoded with exponent 0 (below 2^-126 in magnitude). Lane e < 16 holds
  // escape e as position | exponent << 16, or 0 for an unused slot and for
  // an escape whose exponent is 0 (zeros and BF16 subnormals: exact
  // already).
  // The lanes of row group g (rows g and g + 8) take the escapes of their
  // rows, the groups side by side: iteration k gives every group its k-th
  // escape, so a tile's escapes cost as many iterations as the fullest
  // group holds, not one per escape.
  auto fix_escapes = [&](int s, int kt, uint32_t rec) {
    const uint32_t wst = o_w + s * kWeightBytes;
    // whole tiles: all of the tile's escapes; else those in this warp's half
    const bool mine = rec > 0xFFFFu && (kTilePerWarp || ((rec >> 7) & 1u) == static_cast<uint32_t>(hw));
    const unsigned any = __ballot_sync(0xFFFFFFFFu, mine);
    if (!any) return;
    const uint32_t grp = (rec >> 8) & 7u;  // row group of this lane's escape
    const unsigned b1 = __ballot_sync(0xFFFFFFFFu, grp & 1u), b2 = __ballot_sync(0xFFFFFFFFu, grp & 2u),
                   b4 = __ballot_sync(0xFFFFFFFFu, grp & 4u);
    unsigned pending = any & ((g & 1) ? b1 : ~b1) & ((g & 2) ? b2 : ~b2) & ((g & 4) ? b4 : ~b4);
    const unsigned rounds = __reduce_max_sync(0xFFFFFFFFu, static_cast<unsigned>(__popc(pending)));
    for (unsigned k = 0; k < rounds; ++k) {
      const int e = pending ? __ffs(pending) - 1 : 31;  // lane 31 holds no escape
      pending &= pending - 1;
      const uint32_t erec = __shfl_sync(0xFFFFFFFFu, rec, e);
      const uint32_t eex = erec >> 16;
      const uint32_t r = (erec >> 8) & 255u, c = erec & 255u;
      if (erec > 0xFFFFu) {
        const uint32_t L = 2 * (16 * jw + r) + (c >> 7), bc = c & 127;  // 128-byte line of the sm byte
        const uint32_t smb = sm8[wst + L * 128 + (((bc >> 4) ^ (L & 7)) << 4) + (bc & 15)];
        const float wv = bf16_bits_to_float(bf16_bits(smb, eex));
        // x of batch rows 2t, 2t + 1 (+ 8 nb) at tile column c
        const uint32_t xc = XRES ? o_x + kt * (kTileCols * 2) + c * 2 : o_x + s * xstage + jw * B * kXRowStride + c * 2;
        const uint32_t xstep = XRES ? xrs : kXRowStride;
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
          const int b0 = nb * 8 + 2 * t;
          const float x0 = (b0 < B) ? bf16_bits_to_float(lds_at<uint16_t>(sm8, xc + b0 * xstep)) : 0.f;
          const float x1 = (b0 + 1 < B) ? bf16_bits_to_float(lds_at<uint16_t>(sm8, xc + (b0 + 1) * xstep)) : 0.f;
          if (r >= 8) {
            acc[0][nb][2] = fmaf(wv, x0, acc[0][nb][2]);
            acc[0][nb][3] = fmaf(wv, x1, acc[0][nb][3]);
          } else {
            acc[0][nb][0] = fmaf(wv, x0, acc[0][nb][0]);
            acc[0][nb][1] = fmaf(wv, x1, acc[0][nb][1]);
          }
        }
      }
    }
  };

  // Tile row tr ends: deposit this warp's partial in reduction buffer
  // (local row index & 1) for the reducer warp. A warp waits only to reuse
  // a buffer whose previous row the reducer has not summed yet.
  auto finish_row = [&](int tr) {
    const int lr = tr - tr_first;
    const int pb = lr & 1;
    const uint32_t use = static_cast<uint32_t>(lr >> 1) & 1u;
    if (ok && !mbar_wait(&redfree[pb], use ^ 1u)) ok = false;
    if (ok) {
      float* rw = red + (pb * kCons + warp) * 16 * B;
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        const int b0 = nb * 8 + 2 * t;
        if (b0 < B) {
          rw[g * B + b0] = acc[0][nb][0] + acc[1][nb][0];
          rw[(g + 8) * B + b0] = acc[0][nb][2] + acc[1][nb][2];
        }
        if (b0 + 1 < B) {
          rw[g * B + b0 + 1] = acc[0][nb][1] + acc[1][nb][1];
          rw[(g + 8) * B + b0 + 1] = acc[0][nb][3] + acc[1][nb][3];
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&deposited[pb]);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) acc[h][nb][0] = acc[h][nb][1] = acc[h][nb][2] = acc[h][nb][3] = 0.f;
  };

  const int fb_shift = tstart & 3;  // the fallback indices of a record slot start at its 4-aligned tile

  if constexpr (WIDE) {
    // Group c = warp / 4 takes stages c, c + kWideGroups, c + 2 kWideGroups,
    // ...; warp w multiplies tile w % 4 of each. Before each of its tiles a
    // warp deposits its partials of the rows that end before the tile
    // (zeros for rows it has no tile in), then settles the escape-record
    // groups in order: it waits for each and arrives on its empty barrier
    // once, the groups whose stages it skips included (a warp takes at most
    // one stage of a group). Rows come first, so that no warp waits for
    // records or weights while another needs its partial. Every warp
    // deposits every row, in order: its waits on a reduction buffer's
    // barrier then stay within one phase of the reducer, which is all a
    // parity wait can tell apart. A stage's slot is released by the group's
    // 4 warps once its data has landed.
    constexpr int kG = kWideGroups;
    const int grp = warp >> 2;
    const int tr_end = (tend > tstart) ? (tend - 1) / KT : tr_first - 1;
    const int ngroups = (nstages + kRecStages - 1) / kRecStages;
    int row_next = tr_first;  // the next row this warp deposits
    int rg = 0, rslot = 0;    // the next record group this warp settles, its slot
    uint32_t rph = 0u;        // parity of that slot's phase
    auto next_group = [&]() {
      ++rg;
      if (++rslot == kRS) {
        rslot = 0;
        rph ^= 1u;
      }
    };
    auto settle_records = [&](int upto) {
      while (rg < upto) {
        if (ok) ok = mbar_wait(&rec_full[rslot], rph);
        __syncwarp();
        if (lane == 0) mbar_arrive(&rec_empty[rslot]);
        next_group();
      }
    };
    grid_dependency_wait();
    if (!mbar_wait((K & 7) ? xready : xbar, 0)) ok = false;
    int s = grp;  // stage slot, i % S (S > kG)
    uint32_t ph = 0u;
    int tile0 = tstart + grp * kStage;
    int tr0 = tile0 / KT, kt0 = tile0 - tr0 * KT;
    for (int i = grp; i < nstages; i += kG) {
      const bool have = jw < min(kStage, tend - tile0);
      int kt_w = kt0 + jw, tr_w = tr0;
      while (kt_w >= KT) {
        kt_w -= KT;
        ++tr_w;
      }
      if (have)
        while (row_next < tr_w) finish_row(row_next++);
      const int R = i / kRecStages;
      settle_records(R);
      if (ok) ok = mbar_wait(&rec_full[rslot], rph);
      int fbi_w = -1;
      uint32_t rec_w = 0u;
      if (have) {
        const uint32_t rb = o_rec + rslot * kRecSlotBytes;
        const int lt = (i - R * kRecStages) * kStage + jw;
        fbi_w = lds_at<int>(sm8, rb + kRecFbOffset + (lt + fb_shift) * 4);
        if (lane < kEscapeBudget) {
          const uint32_t pos = lds_at<uint16_t>(sm8, rb + kRecPosOffset + lt * 32 + lane * 2);
          const uint32_t ex = lds_at<uint8_t>(sm8, rb + kRecEscOffset + lt * 16 + lane);
          if (pos != kNoEscape) rec_w = pos | (ex << 16);
        }
        const int seg = segment_of(a.m, tr_w);
        if (seg != cur_seg) {
          const uint4 v = seg_tab[seg];
          tab[0] = v.x;
          tab[1] = v.y;
          tab[2] = v.z;
          tab[3] = v.w;
          pad_inf = (K & (kTileCols - 1)) && (v.x & 0xFFu) == 0xFFu;
          cur_seg = seg;
        }
      }
      // The groups take the stages in turn, so this group never waited on
      // stage i - S of its slot, and a parity wait for stage i would pass on
      // that stage's phase if it had not landed yet. First wait (by parity)
      // until stage i - S is consumed: that phase's predecessor, stage
      // i - 2S, is consumed already (stage i - S was issued, as stage i - 5
      // was, in order), and stage i is not, so the parity tells. Then stage
      // i - S has landed, and the wait for stage i is exact too.
      if (ok && i >= S) ok = mbar_wait(&empty[s], ph ^ 1u);
      if (ok) ok = mbar_wait(&full[s], ph);
      if (have && ok) {
        if (fbi_w < 0 && !pad_inf) {
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            decode_mma(s, kt_w, h);
            if (h == 0) fix_escapes(s, kt_w, rec_w);
          }
        } else {
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            load_frags(s, kt_w, fbi_w, h);
            mma_tile(s, kt_w, h);
            if (h == 0 && fbi_w < 0) fix_escapes(s, kt_w, rec_w);
          }
        }
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&empty[s]);
        mbar_arrive(&rec_empty[rslot]);
      }
      next_group();
      s += kG;
      if (s >= S) {
        s -= S;
        ph ^= 1u;
      }
      tile0 += kG * kStage;
      kt0 += kG * kStage;
      while (kt0 >= KT) {
        kt0 -= KT;
        ++tr0;
      }
    }
    while (row_next <= tr_end) finish_row(row_next++);
    settle_records(ngroups);
  } else {
    int s = 0;                 // stage slot of stage i, i % S
    uint32_t ph = 0u;          // parity of its full-barrier phase, (i / S) & 1
    int rq = 0, rslot = 0;     // stage within its record group, the group's slot
    uint32_t rph = 0u;         // parity of the record slot's phase
    int tile0 = tstart;
    int tr0 = tile0 / KT, kt0 = tile0 - tr0 * KT;  // row and column of the stage's first tile
    // The current stage's tile count, this warp's tile column and records.
    int ntl = 0, kt_mine = 0, fbi = -1;
    uint32_t esc_rec = 0u;  // this lane's escape record (fix_escapes)

    // Waits for stage i's records and weights; with `predecode`, decodes this
    // warp's tile of it (its first half, with 8-tile stages) into frag0 / frag1.
    auto fetch_stage = [&](bool predecode) {
      ntl = min(kStage, tend - tile0);
      fbi = -1;
      esc_rec = 0u;
      if (!RAW) {
        if (rq == 0 && ok) ok = mbar_wait(&rec_full[rslot], rph);
        if (jw < ntl) {
          const uint32_t rb = o_rec + rslot * kRecSlotBytes;
          const int lt = rq * kStage + jw;
          fbi = lds_at<int>(sm8, rb + kRecFbOffset + (lt + fb_shift) * 4);
          if (lane < kEscapeBudget) {
            const uint32_t pos = lds_at<uint16_t>(sm8, rb + kRecPosOffset + lt * 32 + lane * 2);
            const uint32_t ex = lds_at<uint8_t>(sm8, rb + kRecEscOffset + lt * 16 + lane);
            if (pos != kNoEscape) esc_rec = pos | (ex << 16);
          }
        }
      }
      if (ok) ok = mbar_wait(&full[s], ph);
      kt_mine = kt0 + jw;
      int tr_mine = tr0;
      while (kt_mine >= KT) {
        kt_mine -= KT;
        ++tr_mine;
      }
      if (!RAW) {
        const int seg = segment_of(a.m, tr_mine);
        if (seg != cur_seg) {
          const uint4 v = seg_tab[seg];
          tab[0] = v.x;
          tab[1] = v.y;
          tab[2] = v.z;
          tab[3] = v.w;
          pad_inf = (K & (kTileCols - 1)) && (v.x & 0xFFu) == 0xFFu;
          cur_seg = seg;
        }
      }
      if (predecode && jw < ntl && ok) load_frags(s, kt_mine, fbi, 0);
    };

    // The weights do not depend on the previous kernel in the stream: decode
    // this warp's first tile while that kernel finishes, then wait for it
    // (griddepcontrol.wait) before touching x, y or the workspace.
    // (8-tile stages do not: fragments live across the loop would cost the
    // per-group decode its registers; measured slower)
    constexpr bool kPredecodeFirst = !FULL;
    if (nstages > 0) fetch_stage(kPredecodeFirst);
    grid_dependency_wait();
    if (XRES && !mbar_wait((K & 7) ? xready : xbar, 0)) ok = false;

    for (int i = 0; i < nstages; ++i) {
      // Tile rows end at stage positions pe, pe + KT, ... (column KT - 1);
      // the CTA's last tile (position ntl - 1 of its last stage) ends its
      // last row. This warp finishes the rows that end before its tile jw,
      // multiplies tile jw, then finishes the rows that end at or after it,
      // in the order of the tile sequence.
      {
        int pe = KT - 1 - kt0;  // first row end in this stage
        int tr = tr0;
        while (pe < jw && pe < ntl) {
          finish_row(tr);
          ++tr;
          pe += KT;
        }
        if (jw < ntl && ok) {
          if (FULL) {
            // half 0 was decoded by fetch_stage for the first stage
            const bool plain = fbi < 0 && !pad_inf;
            // The two halves run as a loop, not unrolled: one copy of the
            // decode in the instruction cache. The escape products come
            // after half 0, so that their record is dead during half 1.
            if (plain) {
  #pragma unroll 1
              for (int h = 0; h < 2; ++h) {
                decode_mma(s, kt_mine, h);
                if (h == 0) fix_escapes(s, kt_mine, esc_rec);
              }
            } else {
  #pragma unroll 1
              for (int h = 0; h < 2; ++h) {
                if (!(kPredecodeFirst && i == 0 && h == 0)) load_frags(s, kt_mine, fbi, h);
                mma_tile(s, kt_mine, h);
                if (h == 0 && fbi < 0) fix_escapes(s, kt_mine, esc_rec);
              }
            }
          } else {
            mma_tile(s, kt_mine, 0);
            if (!RAW && fbi < 0) fix_escapes(s, kt_mine, esc_rec);
          }
        }
        while (pe < ntl) {
          finish_row(tr);
          ++tr;
          pe += KT;
        }
        // pe is now the first row end past the stage: the stage's last tile
        // ended a row iff pe - KT == ntl - 1
        if (i == nstages - 1 && pe - KT != ntl - 1) finish_row(tr);
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&empty[s]);
        if (!RAW && (rq == kRecStages - 1 || i == nstages - 1)) mbar_arrive(&rec_empty[rslot]);
      }
      if (++s == S) {
        s = 0;
        ph ^= 1u;
      }
      if (++rq == kRecStages) {
        rq = 0;
        if (++rslot == kRS) {
          rslot = 0;
          rph ^= 1u;
        }
      }
      tile0 += kStage;
      kt0 += kStage;
      while (kt0 >= KT) {
        kt0 -= KT;
        ++tr0;
      }
      // 8-tile stages decode in decode_mma (group by group) from the second
      // stage on; 4-tile stages decode here, ahead of the stage's row ends
      if (i + 1 < nstages) fetch_stage(!FULL);
    }

  }
}

cudaError_t launch_gemv(bool raw, const CUtensorMap& map0, const CUtensorMap& map1, const GemvArgs& a, int nblocks,
                        size_t smem, cudaStream_t stream, bool pdl) {
  using Kernel = void (*)(const CUtensorMap, const CUtensorMap, const GemvArgs);
  // [batch blocks][kind: SE12 4-tile, SE12 8-tile, dense][x resident];
  // 8-tile stages always hold x resident
  static const Kernel table[2][3][2] = {
      {{gemv_kernel<1, false, false, false, false, false>, gemv_kernel<1, false, true, false, false, false>},
       {nullptr, gemv_kernel<1, false, true, true, false, false>},
       {gemv_kernel<1, true, false, false, false, false>, gemv_kernel<1, true, true, false, false, false>}},
      {{gemv_kernel<2, false, false, false, false, false>, gemv_kernel<2, false, true, false, false, false>},
       {nullptr, gemv_kernel<2, false, true, true, false, false>},
       {gemv_kernel<2, true, false, false, false, false>, gemv_kernel<2, true, true, false, false, false>}}};
  // with the peer all-reduce (SE12 only): [batch blocks][4-tile, 8-tile][x resident]
  static const Kernel table_ar[2][2][2] = {
      {{gemv_kernel<1, false, false, false, true, false>, gemv_kernel<1, false, true, false, true, false>},
       {nullptr, gemv_kernel<1, false, true, true, true, false>}},
      {{gemv_kernel<2, false, false, false, true, false>, gemv_kernel<2, false, true, false, true, false>},
       {nullptr, gemv_kernel<2, false, true, true, true, false>}}};
  // the wide layout (SE12, x resident, no all-reduce, batch <= 8: at 96
  // registers the two-block accumulators spill)
  static const Kernel table_wide[2] = {gemv_kernel<1, false, true, false, false, kLayoutWide>, nullptr};
  // SE12 without the all-reduce, one CTA per SM: [batch blocks][4-tile,
  // 8-tile][x resident]; the configurations the launch table picks with one
  // CTA per SM (4-tile stages at batch <= 8 never are: they run the classic build)
  static const Kernel table_solo[2][2][2] = {
      {{nullptr, nullptr}, {nullptr, gemv_kernel<1, false, true, true, false, kLayoutSolo>}},
      {{gemv_kernel<2, false, false, false, false, kLayoutSolo>, gemv_kernel<2, false, true, false, false, kLayoutSolo>},
       {nullptr, gemv_kernel<2, false, true, true, false, kLayoutSolo>}}};
  const int kind = raw ? 2 : (a.full_tiles ? 1 : 0);
  const int blocks = nblocks == 1 ? 0 : 1;
  const bool ar = a.peers.world > 1;
  if (ar && raw) return cudaErrorInvalidValue;
  if (a.wide && (raw || ar || a.full_tiles || !a.x_resident || a.stages <= kWideGroups)) return cudaErrorInvalidValue;
  const Kernel solo =
      (!a.wide && !raw && !ar && smem > kCoResidentSmem) ? table_solo[blocks][kind][a.x_resident ? 1 : 0] : nullptr;
  const Kernel kernel = a.wide ? table_wide[blocks]
                        : solo ? solo
                        : ar   ? table_ar[blocks][kind][a.x_resident ? 1 : 0]
                               : table[blocks][kind][a.x_resident ? 1 : 0];
  if (!kernel) return cudaErrorInvalidValue;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.grid);
  cfg.blockDim = dim3(gemv_threads(a.wide != 0));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, map0, map1, a);
}

}  // namespace se12
