// Fused SE12 decode + GEMV for sm_100a:  y[B, N] = x[B, K] . W[N, K]^T
//
// Replaces the reference's lws_gemv_se12 (src/lws/adapters/cuda/kernels/
// gemv_se12.cu:50-142), which runs one warp per (row, batch) with byte loads
// and re-reads the weights once per batch element. Design here:
//
// * Stream-K over the tile sequence. The matrix is the linear sequence of
//   its T tiles in memory order (tile row major, 16x256 weights each). CTA c
//   owns the contiguous range [T*c/G, T*(c+1)/G). Rows of tiles entirely
//   inside a range are written directly; a tile row split between CTAs is
//   finished by the last contributor, which sums the partials in CTA order
//   (deterministic, no floating-point atomics).
// * Warp-specialised pipeline, one tile per stage: a producer warp moves the
//   tile's sm and ec bytes with 2-D TMA loads (128-byte swizzle), the escape
//   slots / escape positions / x slice with 1-D bulk copies, all completing
//   on one mbarrier; four consumer warps each take a 64-column quarter.
//   Fallback tiles are fetched raw (8 KB) instead of sm+ec.
// * Decode in registers straight into mma.sync fragments: per pair of
//   weights one byte-permute (sign|mantissa), one lookup of the ec byte in a
//   lane-replicated 256-entry pair table (conflict-free), one lop3. Escaped
//   weights decode to +0 in the fragment and are added exactly afterwards
//   (w_escaped * x in fp32) from the per-tile escape position list.
// * bf16 m16n8k16 tensor-core MMA with fp32 accumulation; batch padded to
//   multiples of 8. The MMA's k order is permuted per thread so that each
//   thread's operands are 16 contiguous weights of one row (the same
//   permutation is applied to x), and MMA rows are mapped to tile rows by a
//   3-bit reversal so that every shared-memory read is bank-conflict free.
//
// The dense BF16 baseline (RAW = true) runs the same pipeline over a plain
// row-major BF16 matrix (the reference's lws_gemv_raw_bf16,
// src/lws/adapters/cuda/kernels/gemv_raw_bf16.cu:18-56).
#include "se12_device.cuh"
#include "se12_internal.h"

namespace se12 {

__device__ __forceinline__ int bitrev3(int v) { return ((v & 1) << 2) | (v & 2) | ((v >> 2) & 1); }

__device__ __forceinline__ int range_start(int c, int tiles, int grid) {
  return static_cast<int>((static_cast<long long>(tiles) * c) / grid);
}

// CTA whose range contains tile i.
__device__ __forceinline__ int tile_owner(int i, int tiles, int grid) {
  return static_cast<int>(((static_cast<long long>(i) + 1) * grid - 1) / tiles);
}

// Offset of pair-table row `byte k of w` for this lane: byte * 128 + lane * 4.
template <int K>
__device__ __forceinline__ uint32_t lut_offset(uint32_t w, uint32_t lane4) {
  const uint32_t shifted = (K == 0) ? (w << 7) : (w >> (8 * K - 7));
  return (shifted & 0x7F80u) | lane4;
}

__device__ __forceinline__ uint32_t lds32(const uint8_t* base, uint32_t offset) {
  return *reinterpret_cast<const uint32_t*>(base + offset);
}

// Decodes the 16 weights (one row, 16 contiguous columns) of this thread:
// sm bytes in `s`, ec bytes in `e`. Writes fragment halves for MMA j = 0..3:
// lo[j] = weights (4j, 4j+1), hi[j] = weights (4j+2, 4j+3).
__device__ __forceinline__ void decode_row16(uint4 s, uint2 e, const uint8_t* lut, uint32_t lane4, uint32_t (&lo)[4],
                                             uint32_t (&hi)[4]) {
  const uint32_t sw[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t ew = (j < 2) ? e.x : e.y;
    uint32_t t0, t1;
    if ((j & 1) == 0) {
      t0 = lds32(lut, lut_offset<0>(ew, lane4));
      t1 = lds32(lut, lut_offset<1>(ew, lane4));
    } else {
      t0 = lds32(lut, lut_offset<2>(ew, lane4));
      t1 = lds32(lut, lut_offset<3>(ew, lane4));
    }
    lo[j] = pair_word(__byte_perm(sw[j], 0, 0x1100), t0);
    hi[j] = pair_word(__byte_perm(sw[j], 0, 0x3322), t1);
  }
}

// Zeroes the halves of this thread's weight pairs and x pairs whose column
// is >= `valid` (last, partial k-tile of a matrix with K % 256 != 0).
__device__ __forceinline__ uint32_t keep_pair(uint32_t w, int col, int valid) {
  const uint32_t lo = (col < valid) ? 0x0000FFFFu : 0u;
  const uint32_t hi = (col + 1 < valid) ? 0xFFFF0000u : 0u;
  return w & (lo | hi);
}

template <int NB, bool RAW>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const __grid_constant__ CUtensorMap map0,
                                                            const __grid_constant__ CUtensorMap map1,
                                                            const __grid_constant__ GemvArgs a) {
  constexpr int kRedCols = 8 * NB;
  extern __shared__ uint8_t smem_dynamic[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dynamic) + 1023) & ~uintptr_t(1023));

  const int S = a.stages;
  const int xstage = (a.batch * kXRowStride + 127) / 128 * 128;
  uint8_t* wbuf = base;
  uint8_t* p = base + S * kStageWeightBytes;
  uint8_t* lut = p;
  if (!RAW) p += kLutBytes;
  uint8_t* xbuf = p;
  p += S * xstage;
  uint8_t* escbuf = p;
  p += S * 16;
  uint16_t* posbuf = reinterpret_cast<uint16_t*>(p);
  p += S * 32;
  int* meta = reinterpret_cast<int*>(p);
  p += S * 16;
  float* red = reinterpret_cast<float*>(p);
  p += kConsumerWarps * 16 * kRedCols * 4;
  uint64_t* full = reinterpret_cast<uint64_t*>(p);
  p += S * 8;
  uint64_t* empty = reinterpret_cast<uint64_t*>(p);
  p += S * 8;
  int* flag = reinterpret_cast<int*>(p);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int KT = a.m.tile_cols;
  const int T = a.m.tiles;
  const int K = a.m.cols;
  const int start = range_start(blockIdx.x, T, a.grid);
  const int end = range_start(blockIdx.x + 1, T, a.grid);
  const int n = end - start;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_barrier_init();
  }
  if (!RAW) {
    uint32_t* lut32 = reinterpret_cast<uint32_t*>(lut);
    for (int i = tid; i < 256 * kLutCopies; i += blockDim.x) lut32[i] = pair_entry(a.m.codebook, i >> 5);
  }
  __syncthreads();
  grid_launch_dependents();

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    const uint64_t pol_w = policy_evict_first();
    const uint64_t pol_x = policy_evict_last();
    if (lane == 0) {
      prefetch_tmap(&map0);
      if (!RAW) prefetch_tmap(&map1);
    }
    auto x_bytes = [&](int kt) -> uint32_t {
      // the last slice of a row is rounded up to 16 bytes; the caller pads
      // x rows to a multiple of 8 elements and the columns >= K are masked
      const int valid = min(kTileCols, K - kt * kTileCols);
      return (static_cast<uint32_t>(valid) * 2u + 15u) & ~15u;
    };
    auto issue_weights = [&](int i) {
      const int tile = start + i, s = i % S;
      const int tr = tile / KT, kt = tile - tr * KT;
      if (lane == 0) {
        uint8_t* w = wbuf + s * kStageWeightBytes;
        uint32_t wbytes;
        int fb = -1;
        if (RAW) {
          wbytes = kStageWeightBytes;
        } else {
          const uint32_t bits = a.m.bitmap[tile >> 3];
          if ((bits >> (7 - (tile & 7))) & 1u) fb = a.m.fallback_index[tile];
          wbytes = (fb >= 0) ? kStageWeightBytes : (6144 + 48);
        }
        meta[s * 4] = fb;
        mbar_arrive_expect_tx(&full[s], wbytes + static_cast<uint32_t>(a.batch) * x_bytes(kt));
        if (RAW) {
#pragma unroll
          for (int c = 0; c < 4; ++c) tma_load_2d(w + c * 2048, &map0, kt * kTileCols + c * 64, tr * kTileRows, &full[s], pol_w);
        } else if (fb >= 0) {
          bulk_load(w, a.m.fallback_raw + static_cast<size_t>(fb) * kTileSize, kStageWeightBytes, &full[s], pol_w);
        } else {
          tma_load_2d(w, &map0, 0, tile * kTileRows, &full[s], pol_w);
          tma_load_2d(w + 2048, &map0, 128, tile * kTileRows, &full[s], pol_w);
          tma_load_2d(w + 4096, &map1, 0, tile * kTileRows, &full[s], pol_w);
          bulk_load(escbuf + s * 16, a.m.esc + static_cast<size_t>(tile) * 16, 16, &full[s], pol_w);
          bulk_load(posbuf + s * 16, a.m.escape_pos + static_cast<size_t>(tile) * 16, 32, &full[s], pol_w);
        }
      }
      __syncwarp();
    };
    auto issue_x = [&](int i) {
      const int tile = start + i, s = i % S;
      const int kt = tile % KT;
      if (lane < a.batch) {
        bulk_load(xbuf + s * xstage + lane * kXRowStride, a.x + static_cast<size_t>(lane) * a.ldx + kt * kTileCols,
                  x_bytes(kt), &full[s], pol_x);
      }
      __syncwarp();
    };
    const int prologue = min(n, S);
    for (int i = 0; i < prologue; ++i) issue_weights(i);
    grid_dependency_wait();  // x is produced by the previous kernel in the stream
    for (int i = 0; i < prologue; ++i) issue_x(i);
    for (int i = prologue; i < n; ++i) {
      const int s = i % S;
      const uint32_t ph = static_cast<uint32_t>(i / S) & 1u;
      if (!mbar_wait(&empty[s], ph ^ 1u)) break;
      issue_weights(i);
      issue_x(i);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  grid_dependency_wait();
  const int q = warp;                // 64-column quarter of every tile
  const int g = lane >> 2, t = lane & 3;
  const int rg = RAW ? g : bitrev3(g);  // tile rows rg and rg + 8 of this thread
  const int X = rg & 7;                 // 128-byte swizzle phase of those rows
  const uint32_t lane4 = static_cast<uint32_t>(lane) << 2;
  const int ctid = tid;              // 0..127 among consumer threads

  float acc[NB][4];
#pragma unroll
  for (int nb = 0; nb < NB; ++nb) acc[nb][0] = acc[nb][1] = acc[nb][2] = acc[nb][3] = 0.f;
  bool ok = true;

  for (int i = 0; i < n; ++i) {
    const int tile = start + i, s = i % S;
    const uint32_t ph = static_cast<uint32_t>(i / S) & 1u;
    const int tr = tile / KT, kt = tile - tr * KT;
    if (ok) ok = mbar_wait(&full[s], ph);
    if (ok) {
      const uint8_t* w = wbuf + s * kStageWeightBytes;
      const uint8_t* xs = xbuf + s * xstage;
      const int fb = RAW ? -1 : meta[s * 4];
      uint32_t a0[4], a1[4], a2[4], a3[4];  // fragment registers of MMA j: rows rg (a0, a2), rg + 8 (a1, a3)
      if (RAW) {
        const uint8_t* c0 = w + q * 2048;
        const uint4 r0a = *reinterpret_cast<const uint4*>(c0 + rg * 128 + (((2 * t) ^ X) << 4));
        const uint4 r0b = *reinterpret_cast<const uint4*>(c0 + rg * 128 + (((2 * t + 1) ^ X) << 4));
        const uint4 r1a = *reinterpret_cast<const uint4*>(c0 + (rg + 8) * 128 + (((2 * t) ^ X) << 4));
        const uint4 r1b = *reinterpret_cast<const uint4*>(c0 + (rg + 8) * 128 + (((2 * t + 1) ^ X) << 4));
        a0[0] = r0a.x; a2[0] = r0a.y; a0[1] = r0a.z; a2[1] = r0a.w;
        a0[2] = r0b.x; a2[2] = r0b.y; a0[3] = r0b.z; a2[3] = r0b.w;
        a1[0] = r1a.x; a3[0] = r1a.y; a1[1] = r1a.z; a3[1] = r1a.w;
        a1[2] = r1b.x; a3[2] = r1b.y; a1[3] = r1b.z; a3[3] = r1b.w;
      } else if (fb >= 0) {
        const uint8_t* r0 = w + rg * 512 + (64 * q + 16 * t) * 2;
        const uint8_t* r1 = w + (rg + 8) * 512 + (64 * q + 16 * t) * 2;
        const uint4 r0a = *reinterpret_cast<const uint4*>(r0), r0b = *reinterpret_cast<const uint4*>(r0 + 16);
        const uint4 r1a = *reinterpret_cast<const uint4*>(r1), r1b = *reinterpret_cast<const uint4*>(r1 + 16);
        a0[0] = r0a.x; a2[0] = r0a.y; a0[1] = r0a.z; a2[1] = r0a.w;
        a0[2] = r0b.x; a2[2] = r0b.y; a0[3] = r0b.z; a2[3] = r0b.w;
        a1[0] = r1a.x; a3[0] = r1a.y; a1[1] = r1a.z; a3[1] = r1a.w;
        a1[2] = r1b.x; a3[2] = r1b.y; a1[3] = r1b.z; a3[3] = r1b.w;
      } else {
        const uint8_t* half = w + (q >> 1) * 2048;
        const int smc = ((4 * (q & 1) + t) ^ X) << 4;
        const uint4 s0 = *reinterpret_cast<const uint4*>(half + rg * 128 + smc);
        const uint4 s1 = *reinterpret_cast<const uint4*>(half + (rg + 8) * 128 + smc);
        const uint8_t* ecb = w + 4096;
        const int ecc = (((2 * q + (t >> 1)) ^ X) << 4) + 8 * (t & 1);
        const uint2 e0 = *reinterpret_cast<const uint2*>(ecb + rg * 128 + ecc);
        const uint2 e1 = *reinterpret_cast<const uint2*>(ecb + (rg + 8) * 128 + ecc);
        decode_row16(s0, e0, lut, lane4, a0, a2);
        decode_row16(s1, e1, lut, lane4, a1, a3);
      }

      const bool partial_k = (kt == KT - 1) && (K & (kTileCols - 1));
      const int valid = K - kt * kTileCols;
      if (partial_k) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int col = 64 * q + 16 * t + 4 * j;
          a0[j] = keep_pair(a0[j], col, valid);
          a1[j] = keep_pair(a1[j], col, valid);
          a2[j] = keep_pair(a2[j], col + 2, valid);
          a3[j] = keep_pair(a3[j], col + 2, valid);
        }
      }

#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        const int row = nb * 8 + g;
        uint4 xa = make_uint4(0, 0, 0, 0), xb = make_uint4(0, 0, 0, 0);
        if (row < a.batch) {
          const uint8_t* xr = xs + row * kXRowStride + (64 * q + 16 * t) * 2;
          xa = *reinterpret_cast<const uint4*>(xr);
          xb = *reinterpret_cast<const uint4*>(xr + 16);
        }
        uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
        if (partial_k) {
#pragma unroll
          for (int m = 0; m < 8; ++m) xw[m] = keep_pair(xw[m], 64 * q + 16 * t + 2 * m, valid);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) mma_bf16_16816(acc[nb], a0[j], a1[j], a2[j], a3[j], xw[2 * j], xw[2 * j + 1]);
      }

      if (!RAW && fb < 0) {
        // Escaped weights of this quarter: decoded as +0 above, added here.
        const uint32_t mypos = (lane < kEscapeBudget) ? posbuf[s * 16 + lane] : kNoEscape;
        const bool mine = (mypos != kNoEscape) && (((mypos & 255u) >> 6) == static_cast<uint32_t>(q));
        unsigned pending = __ballot_sync(0xFFFFFFFFu, mine);
        while (pending) {
          const int e = __ffs(pending) - 1;
          pending &= pending - 1;
          const uint32_t pos = __shfl_sync(0xFFFFFFFFu, mypos, e);
          const int r = static_cast<int>(pos >> 8), c = static_cast<int>(pos & 255u);
          if ((r & 7) == rg) {
            const uint32_t smb = w[(c >> 7) * 2048 + r * 128 + ((((c & 127) >> 4) ^ (r & 7)) << 4) + (c & 15)];
            const float wv = bf16_bits_to_float(bf16_bits(smb, escbuf[s * 16 + e]));
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) {
              const int b0 = nb * 8 + 2 * t;
              const float x0 = (b0 < a.batch) ? bf16_bits_to_float(*reinterpret_cast<const uint16_t*>(xs + b0 * kXRowStride + 2 * c)) : 0.f;
              const float x1 = (b0 + 1 < a.batch) ? bf16_bits_to_float(*reinterpret_cast<const uint16_t*>(xs + (b0 + 1) * kXRowStride + 2 * c)) : 0.f;
              if (r >= 8) {
                acc[nb][2] = fmaf(wv, x0, acc[nb][2]);
                acc[nb][3] = fmaf(wv, x1, acc[nb][3]);
              } else {
                acc[nb][0] = fmaf(wv, x0, acc[nb][0]);
                acc[nb][1] = fmaf(wv, x1, acc[nb][1]);
              }
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    if (kt == KT - 1 || i == n - 1) {
      // ---------------------------------------------------- finish tile row tr
      const bool whole = (tr * KT >= start) && ((tr + 1) * KT <= end);
      const int slot = (tr == start / KT) ? 0 : 1;
      float* rw = red + q * 16 * kRedCols;
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        rw[rg * kRedCols + nb * 8 + 2 * t] = acc[nb][0];
        rw[rg * kRedCols + nb * 8 + 2 * t + 1] = acc[nb][1];
        rw[(rg + 8) * kRedCols + nb * 8 + 2 * t] = acc[nb][2];
        rw[(rg + 8) * kRedCols + nb * 8 + 2 * t + 1] = acc[nb][3];
        acc[nb][0] = acc[nb][1] = acc[nb][2] = acc[nb][3] = 0.f;
      }
      named_barrier(1, kConsumerWarps * 32);
      const int outs = 16 * a.batch;
      const int stride = 16 * kRedCols;
      float* part = a.partials + (static_cast<size_t>(blockIdx.x) * 2 + slot) * (16 * kRedCols);
      for (int idx = ctid; idx < outs && ok; idx += kConsumerWarps * 32) {
        const int row = idx & 15, b = idx >> 4;
        const float v = ((red[row * kRedCols + b] + red[stride + row * kRedCols + b]) + red[2 * stride + row * kRedCols + b]) +
                        red[3 * stride + row * kRedCols + b];
        if (whole) {
          const int grow = tr * kTileRows + row;
          if (grow < a.m.rows) a.y[static_cast<size_t>(b) * a.ldy + grow] = v;
        } else {
          part[b * 16 + row] = v;
        }
      }
      if (!whole) {
        __threadfence();
        named_barrier(1, kConsumerWarps * 32);
        const int c_lo = tile_owner(tr * KT, T, a.grid);
        const int c_hi = tile_owner((tr + 1) * KT - 1, T, a.grid);
        if (ctid == 0) {
          int last = 0;
          if (ok) last = (atomicAdd(&a.counters[tr], 1) == c_hi - c_lo);
          *flag = last;
        }
        named_barrier(1, kConsumerWarps * 32);
        if (*flag) {
          __threadfence();
          for (int idx = ctid; idx < outs; idx += kConsumerWarps * 32) {
            const int row = idx & 15, b = idx >> 4;
            float v = 0.f;
            for (int c = c_lo; c <= c_hi; ++c) {
              const int cslot = (range_start(c, T, a.grid) / KT == tr) ? 0 : 1;
              v += __ldcg(a.partials + (static_cast<size_t>(c) * 2 + cslot) * (16 * kRedCols) + b * 16 + row);
            }
            const int grow = tr * kTileRows + row;
            if (grow < a.m.rows) a.y[static_cast<size_t>(b) * a.ldy + grow] = v;
          }
          if (ctid == 0) a.counters[tr] = 0;
        }
      }
      named_barrier(1, kConsumerWarps * 32);
    }
  }
}

cudaError_t launch_gemv(bool raw, const CUtensorMap& map0, const CUtensorMap& map1, const GemvArgs& a, int nblocks,
                        size_t smem, cudaStream_t stream, bool pdl) {
  void (*kernel)(const CUtensorMap, const CUtensorMap, const GemvArgs) = nullptr;
  if (raw) {
    kernel = (nblocks == 1) ? gemv_kernel<1, true> : gemv_kernel<2, true>;
  } else {
    kernel = (nblocks == 1) ? gemv_kernel<1, false> : gemv_kernel<2, false>;
  }
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.grid);
  cfg.blockDim = dim3(kGemvThreads);
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
