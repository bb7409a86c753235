// Persistent chain kernel for sm_100a: a whole sequence of GEMVs (for example
// every projection of one decode step, in order) in one launch.
//
// Why: a decode step is a chain of dependent GEMVs (each one's input is
// computed from the previous one's output), most of them a few microseconds
// of HBM traffic. Launched one by one, each pays a fixed cost for its grid to
// fill, drain and hand over to the next kernel -- about as much as the data
// time of a small projection. Here one grid of one CTA per SM walks all the
// GEMVs; only the reads of x wait for the previous GEMV, while the weight
// stream of the next GEMV is already in flight.
//
// Work split. Each GEMV's tiles (16 x 256 weights, tile-row-major order) are
// cut into one contiguous range per CTA (a host table), whole tile rows per
// CTA unless an even split of the tiles is clearly shorter; each CTA's range
// is cut evenly over its consumer warps. A warp accumulates its tiles row by
// row in mma.sync accumulators. A tile row held entirely by one warp is
// written to y by that warp. A row shared by several warps of the CTA is
// stored by each as a share in shared memory; the warp that arrives last on
// the row's counter (tiles summed so far) adds the shares in warp order --
// deterministic, no floating-point atomics, nobody waits -- and writes y.
// Only when the split cuts a row between CTAs do the CTAs' sums of that row
// go through global memory, added by the last CTA to arrive in CTA order.
//
// Pipeline. Every consumer warp owns kChainSlots slots of shared memory and
// issues its own TMA loads into them (one lane): the sm and ec bytes of one
// tile (3-D and 2-D boxes, 128-byte swizzle) and the tile's 64-byte escape
// record, onto the slot's mbarrier. The warp refills a slot as soon as it
// has read it, so its loads run one slot ahead and follow its own position
// in the sequence across GEMV boundaries; no warp waits for another.
//
// x. A control warp copies each GEMV's x (its column range) into shared
// memory once every CTA finished the previous GEMV (global completion
// counters that grow by the grid size per launch), zeroes the columns past
// K and releases the consumers. Its columns, like the weights', decode
// straight into mma.sync fragments (decode8, shared with the single-GEMV
// kernel).
//
// The chain's ops may all-reduce their rows over a peer group (tensor
// parallelism with column shards): the warp that completes a row stores it,
// tagged with the op's epoch, into every rank's receive buffer and sums the
// ranks' rows in rank order (the protocol of the single-GEMV kernel).
//
// A dense BF16 variant (RAW) runs the same chain over plain BF16 matrices:
// the comparison baseline.
//
// Every wait is bounded (2 s, or the limit the host set for waits on other
// CTAs and GPUs); on timeout the kernel raises the status word and the
// affected warp stops, after waiting for its own loads in flight.
#include "se12_device.cuh"
#include "se12_internal.h"

namespace se12 {

// Record flags (word 0 of a tile's 16-word record).
constexpr uint32_t kRecFallback = 0x80000000u;   // raw tile: bits 0..29 = fallback index
constexpr uint32_t kRecPadPatch = 0x40000000u;   // last tile column of a segment whose padding decodes to inf

// ---------------------------------------------------------------- records

// One warp per tile: the tile's record, 16 words. Word e < 16 holds the
// e-th escaped weight as position | exponent << 16 (position = 16 r + c...
// the tile-flat index r * 256 + c), or 0 for an unused slot and for an
// escape whose true exponent is 0 (it decodes exactly without a fix). A
// fallback tile's word 0 is kRecFallback | its rank among fallback tiles.
// Needs the derived tables of se12_matrix_prepare.
__global__ void prepare_tile_records(const __grid_constant__ MatrixView m, uint32_t* __restrict__ records) {
  const int warps = blockDim.x >> 5;
  const int tile = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (tile >= m.tiles || lane >= kEscapeBudget) return;
  const int fbi = m.fallback_index[tile];
  uint32_t w = 0;
  if (fbi >= 0) {
    w = (lane == 0) ? (kRecFallback | static_cast<uint32_t>(fbi)) : 0u;
  } else {
    const uint32_t pos = m.escape_pos[static_cast<size_t>(tile) * kEscapeBudget + lane];
    const uint32_t ex = m.esc[static_cast<size_t>(tile) * kEscapeBudget + lane];
    if (pos != kNoEscape && ex != 0) w = pos | (ex << 16);
    if (lane == 0) {
      const int tr = tile / m.tile_cols, kt = tile - tr * m.tile_cols;
      const int seg = segment_of(m, tr);
      if (kt == m.tile_cols - 1 && (m.cols & (kTileCols - 1)) && m.codebooks[seg][0] == 255) w |= kRecPadPatch;
    }
  }
  records[static_cast<size_t>(tile) * kEscapeBudget + lane] = w;
}

cudaError_t launch_prepare_records(const MatrixView& m, uint32_t* records, cudaStream_t stream) {
  if (m.tiles == 0) return cudaSuccess;
  const int warps = 8;
  prepare_tile_records<<<(m.tiles + warps - 1) / warps, warps * 32, 0, stream>>>(m, records);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- helpers

__device__ __forceinline__ uint32_t prmt_c(uint32_t a, uint32_t b, uint32_t selector) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(selector));
  return d;
}

__device__ __forceinline__ uint32_t select_bits_c(uint32_t a, uint32_t b, uint32_t m) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xE4;" : "=r"(d) : "r"(a), "r"(b), "r"(m));
  return d;
}

// The 8-weight register decode of the single-GEMV kernel (se12_gemv.cu,
// decode8): sign|mantissa bytes s, codes e (weight i in bits 4i..4i+3),
// table tab[0..3] (table byte of code c in byte c % 4 of tab[c / 4]) ->
// four BF16x2 words, columns (0,1), (2,3), (4,5), (6,7).
__device__ __forceinline__ void chain_decode8(uint2 s, uint32_t e, const uint32_t (&tab)[4], uint32_t (&p)[4]) {
  const uint32_t sel03 = e & 0x77777777u;
  const uint32_t sel47 = __umulhi(sel03, 0x10000u);
  const uint32_t e4 = e << 4;
  const uint32_t hi03 = prmt_c(e4, e, 0xD9C8u);
  const uint32_t hi47 = prmt_c(e4, e, 0xFBEAu);
  const uint32_t x03 = select_bits_c(prmt_c(tab[2], tab[3], sel03), prmt_c(tab[0], tab[1], sel03), hi03);
  const uint32_t x47 = select_bits_c(prmt_c(tab[2], tab[3], sel47), prmt_c(tab[0], tab[1], sel47), hi47);
  const uint32_t lo03 = select_bits_c(s.x, x03, 0x7F7F7F7Fu);
  const uint32_t up03 = select_bits_c(s.x, x03, 0x80808080u);
  const uint32_t lo47 = select_bits_c(s.y, x47, 0x7F7F7F7Fu);
  const uint32_t up47 = select_bits_c(s.y, x47, 0x80808080u);
  p[0] = prmt_c(lo03, up03, 0x5140u);
  p[1] = prmt_c(lo03, up03, 0x7362u);
  p[2] = prmt_c(lo47, up47, 0x5140u);
  p[3] = prmt_c(lo47, up47, 0x7362u);
}

template <typename T>
__device__ __forceinline__ T lds(const uint8_t* smem, uint32_t offset) {
  return *reinterpret_cast<const T*>(smem + offset);
}

// 64-bit flag-free counter helpers: counters grow by the grid size per
// launch; "reached" compares modulo 2^32.
__device__ __forceinline__ unsigned ld_acquire_gpu_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bool counter_reached(const unsigned* p, unsigned target) {
  return static_cast<int>(ld_acquire_gpu_u32(p) - target) >= 0;
}

__device__ __forceinline__ bool wait_counter(const unsigned* p, unsigned target) {
  if (counter_reached(p, target)) return true;
  const unsigned long long start = global_ns();
  while (!counter_reached(p, target)) {
    __nanosleep(32);
    if (peer_wait_expired(start)) {
      raise_status(kStatusWaitTimeout);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ unsigned atom_add_acq_rel_gpu_u32(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ void fence_proxy_async_all() { asm volatile("fence.proxy.async;" ::: "memory"); }

// Waits for an mbarrier phase by polling without suspending the warp: the
// consumers waiting for an op's x have nothing else to do, and a suspended
// warp wakes up later than a polling one. Bounded like mbar_wait.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity) {
  if (mbar_test(bar, parity)) return true;
  const unsigned long long start = global_ns();
  while (!mbar_test(bar, parity)) {
    if (global_ns() - start > kWaitLimitNs) {
      raise_status(kStatusWaitTimeout);
      return false;
    }
  }
  return true;
}

// A CTA's range of n tiles is split over its C consumer warps: warp w holds
// local tiles [n w / C, n (w + 1) / C).
__device__ __forceinline__ int part_start(int n, int w, int C) { return n * w / C; }

// Warp whose part holds local tile t (t < n).
__device__ __forceinline__ int part_owner(int t, int n, int C) { return ((t + 1) * C - 1) / n; }

// CTA whose range holds op tile i: the largest c with starts[c] <= i (an
// empty range never qualifies as the largest, its successor starts at the
// same tile).
__device__ __forceinline__ int cta_owner(const int* st, int G, int i) {
  int lo = 0, hi = G - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(st + mid) <= i) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// ---------------------------------------------------------------- kernel

template <int NB, bool RAW>
__global__ void __launch_bounds__((kChainMaxWarps + 1) * 32, 1) chain_kernel(const __grid_constant__ ChainParams p) {
  constexpr int D = kChainSlots;
  constexpr uint32_t SLOT = RAW ? kChainSlotRaw : kChainSlotSe12;
  constexpr int PB = 16 * 8 * NB;  // floats of one partial row block: [8 NB batch columns][16 rows]
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t pad = (1024u - (smem_addr(smem) & 1023u)) & 1023u;
  const int C = p.consumers;
  const int B = p.batch;
  const int nops = p.n_ops;
  const int G = gridDim.x;
  const int cta = blockIdx.x;
  const uint32_t o_slots = pad;
  const uint32_t o_rec = o_slots + static_cast<uint32_t>(C * D) * SLOT;
  const uint32_t o_x = o_rec + (RAW ? 0u : static_cast<uint32_t>(C * D) * 64u);
  const uint32_t o_part = (o_x + static_cast<uint32_t>(p.x_bytes) + 15u) & ~15u;
  const uint32_t o_bar = o_part + static_cast<uint32_t>(C * 2 * PB) * 4u;
  float* const part_s = reinterpret_cast<float*>(smem + o_part);    // [C][2][PB] warps' shares of shared rows
  uint64_t* const full = reinterpret_cast<uint64_t*>(smem + o_bar);  // [C * D] slot loaded
  uint64_t* const xbar = full + C * D;                               // x copy landed (control warp)
  uint64_t* const xready = xbar + 1;                                  // x of the current op ready
  unsigned* const rowcnt_s = reinterpret_cast<unsigned*>(xready + 1);  // [C][2] tiles summed of a row shared by warps

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < C * D; ++i) mbar_init(&full[i], 1);
    mbar_init(xbar, 1);
    mbar_init(xready, 1);
    for (int i = 0; i < 2 * C; ++i) rowcnt_s[i] = 0u;
    fence_barrier_init();
  }
  __syncthreads();

  // This launch's generation: op j is complete once done[j] reaches
  // (generation + 1) * grid. The last CTA to leave bumps the generation.
  const unsigned gen = *reinterpret_cast<volatile unsigned*>(p.gen);
  const unsigned target = (gen + 1u) * gridDim.x;
  // All-reduce epochs continue the peer group's call counter (shared with
  // se12_gemv_allreduce calls on the same group): op a uses counter + a + 1,
  // and the last CTA to leave adds the chain's all-reduce count.
  const unsigned ar_base = p.n_ar > 0 ? *reinterpret_cast<volatile unsigned*>(p.peers.epoch) : 0u;

  if (warp == C) {
    // ------------------------------------------------------------ control warp: x of every op
    const uint64_t pol_x = policy_evict_last();
    for (int j = 0; j < nops; ++j) {
      const ChainOp* op = p.ops + j;
      bool ok = true;
      // every CTA (this one's consumers included) finished op j - 1: its
      // outputs are visible and this CTA's x buffer is free
      if (j > 0) ok = __all_sync(0xFFFFFFFFu, wait_counter(p.done + (j - 1), target));
      const int width = (op->k1 - op->k0) * kTileCols;
      const int xc = op->x_cols;
      const uint32_t row_bytes = static_cast<uint32_t>((xc + 7) & ~7) * 2u;
      const uint16_t* xsrc = op->x + static_cast<size_t>(op->k0) * kTileCols;
      const int ldx = op->ldx;
      if (ok) {
        fence_proxy_async_all();  // generic accesses (other SMs' y, this CTA's reads of x) before the async copy
        if (lane == 0) mbar_arrive_expect_tx(xbar, row_bytes * static_cast<uint32_t>(B));
        __syncwarp();
        if (lane < B)
          bulk_load(smem + o_x + lane * p.x_stride, xsrc + static_cast<size_t>(lane) * ldx, row_bytes, xbar, pol_x);
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(xbar, static_cast<uint32_t>(j) & 1u));
      }
      if (ok) {
        // columns xc .. width - 1 of every row are zero (the copy brought
        // up to 7 columns past K as the caller left them)
        const int tail = width - xc;
        for (int i = lane; i < B * tail; i += 32) {
          const int b = i / tail, c = xc + (i - b * tail);
          *reinterpret_cast<uint16_t*>(smem + o_x + b * p.x_stride + 2 * c) = 0;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(xready);  // released even on failure: the consumers check the status word
      if (!ok) break;
    }
  } else if (warp < C) {
    // ------------------------------------------------------------ consumer warps
    const int g = lane >> 2, t = lane & 3;
    const uint32_t my_slots = o_slots + static_cast<uint32_t>(warp * D) * SLOT;
    const uint32_t my_recs = o_rec + static_cast<uint32_t>(warp * D) * 64u;
    uint64_t* const my_full = full + warp * D;
    const uint64_t pol_w = policy_evict_first();

    // Per-lane offsets inside a slot (see the file header of se12_gemv.cu
    // for the layout): SE12 sm [16 rows][2 halves][128 B] and ec [16 rows]
    // [128 B] after it, both 128-byte swizzled; group k (columns 32 k + 8 t
    // .. + 7 of rows g and g + 8) sits at off(k) = base_h ^ (32 (k % 4)).
    uint32_t sm_base[2], ec_base;
    {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t L = 2u * g + h;
        sm_base[h] = L * 128u + 8u * (t & 1) + ((((t >> 1) ^ L) & 7u) << 4);
      }
      ec_base = 4096u + g * 128u + 4u * t + (static_cast<uint32_t>(g) << 4);
    }
    // dense tiles: [16 rows][4 chunks of 64 columns][128 B] (3-D box) or
    // [4 chunks][16 rows][128 B] (2-D boxes), 128-byte swizzled
    // x: batch row g (+ 8 nb), column 8 t (+ 32 k, + 256 kt_local)
    const uint32_t x_lane = o_x + static_cast<uint32_t>(g) * p.x_stride + 16u * t;
    const uint32_t x_nb = 8u * p.x_stride;

    // ---- issue side: this warp's tile sequence across ops, kept D tiles
    // ahead of consumption
    // this warp's part of op j: tiles [a, b) of the CTA's range
    auto part_of = [&](int j, int& a, int& b) {
      const int* st = p.starts + static_cast<size_t>(j) * (G + 1);
      const int s = __ldg(st + cta), n = __ldg(st + cta + 1) - s;
      a = s + part_start(n, warp, C);
      b = s + part_start(n, warp + 1, C);
    };
    // the issue side's op fields live in registers, loaded once per op
    int iop = 0, ii = 0, iend = 0;
    int is_k0 = 0, is_w = 1, is_tc = 1, is_r3 = 0;
    const uint32_t* is_rec = nullptr;
    auto seek = [&](int from) {
      iop = from;
      while (iop < nops) {
        part_of(iop, ii, iend);
        if (ii < iend) {
          const ChainOp* op = p.ops + iop;
          is_k0 = op->k0;
          is_w = op->k1 - is_k0;
          is_tc = op->tile_cols;
          is_r3 = op->raw_3d;
          is_rec = op->records;
          return;
        }
        ++iop;
      }
    };
    seek(0);
    uint32_t issued = 0;
    auto issue_next = [&]() {
      if (iop >= nops) return;
      if (lane == 0) {
        const ChainOp* op = p.ops + iop;  // tensor maps: read by the copy engine, not here
        const int tr = ii / is_w;
        const int kt = is_k0 + (ii - tr * is_w);
        const int s = static_cast<int>(issued % D);
        uint8_t* dst = smem + my_slots + s * SLOT;
        uint64_t* bar = &my_full[s];
        if (RAW) {
          mbar_arrive_expect_tx(bar, 8192u);
          if (is_r3) {
            tma_load_3d(dst, &op->sm_map, 0, kt * 4, tr * kTileRows, bar, pol_w);
          } else {
#pragma unroll
            for (int c = 0; c < 4; ++c)
              tma_load_2d(dst + c * 2048, &op->sm_map, kt * kTileCols + c * 64, tr * kTileRows, bar, pol_w);
          }
        } else {
          const int tile = tr * is_tc + kt;
          mbar_arrive_expect_tx(bar, 4096u + 2048u + 64u);
          tma_load_3d(dst, &op->sm_map, 0, 0, tile * kTileRows, bar, pol_w);
          tma_load_2d(dst + 4096, &op->ec_map, 0, tile * kTileRows, bar, pol_w);
          bulk_load(smem + my_recs + s * 64, is_rec + static_cast<size_t>(tile) * kEscapeBudget, 64u, bar, pol_w);
        }
      }
      __syncwarp();
      ++issued;
      if (++ii == iend) seek(iop + 1);
    };
    for (int k = 0; k < D; ++k) issue_next();

    bool ok = true;
    uint32_t consumed = 0;
    float acc[2][NB][4];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) acc[h][nb][0] = acc[h][nb][1] = acc[h][nb][2] = acc[h][nb][3] = 0.f;

    for (int j = 0; j < nops; ++j) {
      const ChainOp* op = p.ops + j;
      const int* const st = p.starts + static_cast<size_t>(j) * (G + 1);
      const int cs = __ldg(st + cta), n = __ldg(st + cta + 1) - cs;  // this CTA's tiles [cs, cs + n)
      const int a = cs + part_start(n, warp, C), b = cs + part_start(n, warp + 1, C);
      // the op's fields (and the decode table of this warp's first tile),
      // loaded before its x is ready: their latency hides under that wait
      const int k0 = op->k0;
      const int W = op->k1 - k0;
      const int N = op->rows;
      const int K = op->cols;
      float* const y = op->y;
      const int ldy = op->ldy;
      const uint16_t* const fbraw = op->fallback_raw;
      const int accumulate = op->accumulate;
      const int ar_index = op->ar_index;
      const bool r3 = RAW && op->raw_3d != 0;
      int seg_end[kMaxSegments];
#pragma unroll
      for (int q = 0; q < kMaxSegments; ++q) seg_end[q] = op->seg_end[q];
      uint32_t tab[4] = {0u, 0u, 0u, 0u};
      int cur_seg = -1;
      if (!RAW && a < b) {
        const int tr0 = a / W;
        int sg = 0;
#pragma unroll
        for (int q = 0; q < kMaxSegments - 1; ++q) sg += (tr0 >= seg_end[q]);
        const uint4 v = *reinterpret_cast<const uint4*>(op->tab[sg]);
        tab[0] = v.x;
        tab[1] = v.y;
        tab[2] = v.z;
        tab[3] = v.w;
        cur_seg = sg;
      }
      if (ok) ok = __all_sync(0xFFFFFFFFu, mbar_wait_spin(xready, static_cast<uint32_t>(j) & 1u));
      if (a < b && ok) {

        int row = a / W;       // current tile row (of the op)
        int seg_first = a;     // op-linear index of this warp's first tile in `row`
        for (int i = a; i < b; ++i) {
          const int tr = i / W;
          const int kt_local = i - tr * W;
          const int kt = k0 + kt_local;
          const int s = static_cast<int>(consumed % D);
          const uint32_t par = (consumed / D) & 1u;
          if (ok) ok = __all_sync(0xFFFFFFFFu, mbar_wait(&my_full[s], par));
          const bool landed = ok;  // the slot's copy arrived (and counts as consumed below)
          if (ok) {
            const uint32_t sb = my_slots + s * SLOT;
            const uint32_t xt = x_lane + static_cast<uint32_t>(kt_local) * 512u;
            float part[2][NB][4];  // the tile's MMAs sum here first (two-level accumulation, see add_acc)
            zero_acc(part);
            if (RAW) {
#pragma unroll
              for (int k = 0; k < 8; ++k) {
                const uint32_t m1 = k >> 1, unit = 4u * (k & 1) + t;
                uint32_t off0;
                if (r3) {
                  const uint32_t line = 4u * g + m1;
                  off0 = line * 128u + ((unit ^ (line & 7u)) << 4);
                } else {
                  off0 = m1 * 2048u + g * 128u + ((unit ^ static_cast<uint32_t>(g)) << 4);
                }
                const uint4 v0 = lds<uint4>(smem, sb + off0);
                const uint4 v1 = lds<uint4>(smem, sb + off0 + (r3 ? 4096u : 1024u));
#pragma unroll
                for (int nb = 0; nb < NB; ++nb) {
                  uint4 xv = make_uint4(0u, 0u, 0u, 0u);
                  if (nb * 8 + g < B) xv = lds<uint4>(smem, xt + nb * x_nb + 64u * k);
                  mma_bf16_16816(part[k & 1][nb], v0.x, v1.x, v0.y, v1.y, xv.x, xv.y);
                  mma_bf16_16816(part[k & 1][nb], v0.z, v1.z, v0.w, v1.w, xv.z, xv.w);
                }
              }
            } else {
              const uint32_t rec = (lane < kEscapeBudget) ? lds<uint32_t>(smem, my_recs + s * 64 + lane * 4) : 0u;
              const uint32_t w0 = __shfl_sync(0xFFFFFFFFu, rec, 0);
              if (__builtin_expect((w0 & kRecFallback) != 0u, 0)) {
                // fallback tile: its raw BF16 bits from global memory
                const uint16_t* raw = fbraw + static_cast<size_t>(w0 & 0x3FFFFFFFu) * kTileSize + 8 * t;
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                  const uint4 v0 = __ldg(reinterpret_cast<const uint4*>(raw + g * kTileCols + 32 * k));
                  const uint4 v1 = __ldg(reinterpret_cast<const uint4*>(raw + (g + 8) * kTileCols + 32 * k));
#pragma unroll
                  for (int nb = 0; nb < NB; ++nb) {
                    uint4 xv = make_uint4(0u, 0u, 0u, 0u);
                    if (nb * 8 + g < B) xv = lds<uint4>(smem, xt + nb * x_nb + 64u * k);
                    mma_bf16_16816(part[k & 1][nb], v0.x, v1.x, v0.y, v1.y, xv.x, xv.y);
                    mma_bf16_16816(part[k & 1][nb], v0.z, v1.z, v0.w, v1.w, xv.z, xv.w);
                  }
                }
              } else {
                int seg = 0;
#pragma unroll
                for (int q = 0; q < kMaxSegments - 1; ++q) seg += (tr >= seg_end[q]);
                if (seg != cur_seg) {
                  const uint4 v = *reinterpret_cast<const uint4*>(op->tab[seg]);
                  tab[0] = v.x;
                  tab[1] = v.y;
                  tab[2] = v.z;
                  tab[3] = v.w;
                  cur_seg = seg;
                }
                const bool patch = (w0 & kRecPadPatch) != 0u;
                const int valid = K - kt * kTileCols;  // columns of this tile inside the matrix
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                  const uint32_t so = sb + (sm_base[k >> 2] ^ (32u * (k & 3)));
                  const uint32_t eo = sb + (ec_base ^ (16u * k));
                  uint32_t e0 = lds<uint32_t>(smem, eo);
                  uint32_t e1 = lds<uint32_t>(smem, eo + 1024u);
                  if (__builtin_expect(patch, 0)) {
                    // padding columns decode with the escape code (exponent 0):
                    // their weights would be inf, x is 0 there
                    uint32_t mask = 0u;
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                      if (32 * k + 8 * t + q >= valid) mask |= 0xFu << (4 * q);
                    e0 |= mask;
                    e1 |= mask;
                  }
                  uint32_t f0[4], f1[4];
                  chain_decode8(lds<uint2>(smem, so), e0, tab, f0);
                  chain_decode8(lds<uint2>(smem, so + 2048u), e1, tab, f1);
#pragma unroll
                  for (int nb = 0; nb < NB; ++nb) {
                    uint4 xv = make_uint4(0u, 0u, 0u, 0u);
                    if (nb * 8 + g < B) xv = lds<uint4>(smem, xt + nb * x_nb + 64u * k);
                    mma_bf16_16816(part[k & 1][nb], f0[0], f1[0], f0[1], f1[1], xv.x, xv.y);
                    mma_bf16_16816(part[k & 1][nb], f0[2], f1[2], f0[3], f1[3], xv.z, xv.w);
                  }
                }
                // exact products of the escaped weights (decoded with
                // exponent 0 above): lane e < 16 holds escape e
                unsigned pending = __ballot_sync(0xFFFFFFFFu, ((rec >> 16) & 0xFFu) != 0u && lane < kEscapeBudget);
                while (pending) {
                  const int e = __ffs(pending) - 1;
                  pending &= pending - 1;
                  const uint32_t er = __shfl_sync(0xFFFFFFFFu, rec, e);
                  const uint32_t pos = er & 0xFFFu, ex = (er >> 16) & 0xFFu;
                  const uint32_t r = pos >> 8, c = pos & 255u;
                  if ((r & 7u) == static_cast<uint32_t>(g)) {
                    const uint32_t L = 2u * r + (c >> 7), bc = c & 127u;
                    const uint32_t smb = smem[sb + L * 128u + ((((bc >> 4) ^ L) & 7u) << 4) + (bc & 15u)];
                    const float wv = __uint_as_float((((smb & 0x80u) << 8) | (ex << 7) | (smb & 0x7Fu)) << 16);
                    const uint32_t xc = o_x + static_cast<uint32_t>(kt_local) * 512u + c * 2u;
#pragma unroll
                    for (int nb = 0; nb < NB; ++nb) {
                      const int b0 = nb * 8 + 2 * t;
                      const float x0 = (b0 < B) ? __uint_as_float(static_cast<uint32_t>(lds<uint16_t>(smem, xc + b0 * p.x_stride)) << 16) : 0.f;
                      const float x1 = (b0 + 1 < B) ? __uint_as_float(static_cast<uint32_t>(lds<uint16_t>(smem, xc + (b0 + 1) * p.x_stride)) << 16) : 0.f;
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
              }
            }
            add_acc(acc, part);  // this tile's MMA sums into the running fp32 sums
          }
          // slot s is read: refill it with the next tile of this warp's sequence
          __syncwarp();
          fence_proxy_async_shared();
          if (landed) ++consumed;
          if (ok) issue_next();

          // ---- row end: the tile row ends here, or this warp's run does
          if (kt_local == W - 1 || i + 1 == b) {
            float v[NB][4];
#pragma unroll
            for (int nb = 0; nb < NB; ++nb)
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                v[nb][q] = acc[0][nb][q] + acc[1][nb][q];
                acc[0][nb][q] = acc[1][nb][q] = 0.f;
              }
            const int row_lo = row * W, row_hi = row_lo + W;
            const bool whole = (seg_first == row_lo) && (i + 1 == row_hi);
            bool emit = ok;
            if (!whole && ok) {
              // A row shared by warps: each stores its share in shared
              // memory and adds its tile count to the row's counter; the last
              // to arrive sums the shares in warp order (deterministic, no
              // float atomics, nobody waits).
              const int which = (row == a / W) ? 0 : 1;  // this warp's first row or its last
              float* mine = part_s + (warp * 2 + which) * PB;
#pragma unroll
              for (int nb = 0; nb < NB; ++nb) {
                const int b0 = nb * 8 + 2 * t;
                mine[b0 * 16 + g] = v[nb][0];
                mine[(b0 + 1) * 16 + g] = v[nb][1];
                mine[b0 * 16 + g + 8] = v[nb][2];
                mine[(b0 + 1) * 16 + g + 8] = v[nb][3];
              }
              const int lo = max(row_lo, cs), hi = min(row_hi, cs + n);  // the row's tiles in this CTA
              const int wf = part_owner(lo - cs, n, C);                   // the first warp holding one
              // the row is wf's first or last row: (wf, 0) or (wf, 1) names it
              const int kf = ((cs + part_start(n, wf, C)) / W == row) ? 0 : 1;
              const unsigned held = static_cast<unsigned>(i + 1 - seg_first);
              __syncwarp();
              unsigned old = 0;
              if (lane == 0) {
                __threadfence_block();
                old = atomicAdd(&rowcnt_s[wf * 2 + kf], held);
                __threadfence_block();
              }
              old = __shfl_sync(0xFFFFFFFFu, old, 0);
              emit = (old + held == static_cast<unsigned>(hi - lo));
              if (emit) {
#pragma unroll
                for (int nb = 0; nb < NB; ++nb)
#pragma unroll
                  for (int q = 0; q < 4; ++q) v[nb][q] = 0.f;
                const int wl = part_owner(hi - 1 - cs, n, C);
                for (int w = wf; w <= wl; ++w) {
                  const int ws = cs + part_start(n, w, C);
                  if (ws == cs + part_start(n, w + 1, C)) continue;  // empty part
                  const float* src = part_s + (w * 2 + ((ws / W == row) ? 0 : 1)) * PB;
#pragma unroll
                  for (int nb = 0; nb < NB; ++nb) {
                    const int b0 = nb * 8 + 2 * t;
                    v[nb][0] += src[b0 * 16 + g];
                    v[nb][1] += src[(b0 + 1) * 16 + g];
                    v[nb][2] += src[b0 * 16 + g + 8];
                    v[nb][3] += src[(b0 + 1) * 16 + g + 8];
                  }
                }
                if (lane == 0) rowcnt_s[wf * 2 + kf] = 0u;  // ready for the next op
                if (lo != row_lo || hi != row_hi) {
                  // the row continues in other CTAs (a stream-K split of the
                  // op): publish this CTA's sum; the last CTA to arrive adds
                  // the CTAs' sums in CTA order
                  float* gp = p.partials + (static_cast<size_t>(cta) * 2 + ((row == cs / W) ? 0 : 1)) * 256;
#pragma unroll
                  for (int nb = 0; nb < NB; ++nb) {
                    const int b0 = nb * 8 + 2 * t;
                    gp[b0 * 16 + g] = v[nb][0];
                    gp[(b0 + 1) * 16 + g] = v[nb][1];
                    gp[b0 * 16 + g + 8] = v[nb][2];
                    gp[(b0 + 1) * 16 + g + 8] = v[nb][3];
                  }
                  __threadfence();
                  __syncwarp();
                  const int cf = cta_owner(st, G, row_lo);
                  const int kc = (__ldg(st + cf) / W == row) ? 0 : 1;
                  unsigned* rc = p.rowcnt + (static_cast<size_t>(j) * G + cf) * 2 + kc;
                  const unsigned mine_tiles = static_cast<unsigned>(hi - lo);
                  unsigned oldg = 0;
                  if (lane == 0) oldg = atom_add_acq_rel_gpu_u32(rc, mine_tiles);
                  oldg = __shfl_sync(0xFFFFFFFFu, oldg, 0);
                  emit = (oldg + mine_tiles == static_cast<unsigned>(W));
                  if (emit) {
                    __threadfence();
#pragma unroll
                    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
                      for (int q = 0; q < 4; ++q) v[nb][q] = 0.f;
                    const int cl = cta_owner(st, G, row_hi - 1);
                    for (int c = cf; c <= cl; ++c) {
                      const int c0 = __ldg(st + c);
                      if (c0 == __ldg(st + c + 1)) continue;  // empty range
                      const float* src = p.partials + (static_cast<size_t>(c) * 2 + ((c0 / W == row) ? 0 : 1)) * 256;
#pragma unroll
                      for (int nb = 0; nb < NB; ++nb) {
                        const int b0 = nb * 8 + 2 * t;
                        v[nb][0] += __ldcg(src + b0 * 16 + g);
                        v[nb][1] += __ldcg(src + (b0 + 1) * 16 + g);
                        v[nb][2] += __ldcg(src + b0 * 16 + g + 8);
                        v[nb][3] += __ldcg(src + (b0 + 1) * 16 + g + 8);
                      }
                    }
                    if (lane == 0) *rc = 0u;  // ready for the next launch
                  }
                }
              }
            }
            if (emit) {
              if (accumulate) {
                // the previous op wrote these rows' other columns
#pragma unroll
                for (int nb = 0; nb < NB; ++nb)
#pragma unroll
                  for (int q = 0; q < 4; ++q) {
                    const int bb = nb * 8 + 2 * t + (q & 1);
                    const int grow = row * kTileRows + g + 8 * (q >> 1);
                    if (bb < B && grow < N) v[nb][q] += __ldcg(y + static_cast<size_t>(bb) * ldy + grow);
                  }
              }
              if (ar_index >= 0) {
                // all-reduce of the row over the peer group: every value with
                // the op's epoch in one 64-bit word into every rank's receive
                // buffer, then all ranks' words summed in rank order
                const PeerArgs& P = p.peers;
                const unsigned epoch = ar_base + static_cast<unsigned>(ar_index) + 1u;
                const size_t slot = static_cast<size_t>(16) * P.rows_cap;
                const size_t base = static_cast<size_t>((epoch & 1u) * P.world) * slot;
                const unsigned long long tag = static_cast<unsigned long long>(epoch) << 32;
                for (int r = 0; r < P.world; ++r) {
                  unsigned long long* dst = P.recv[r] + base + P.rank * slot;
#pragma unroll
                  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                      const int bb = nb * 8 + 2 * t + (q & 1);
                      const int grow = row * kTileRows + g + 8 * (q >> 1);
                      if (bb < B && grow < N)
                        st_word_sys(dst + static_cast<size_t>(bb) * P.rows_cap + grow, tag | __float_as_uint(v[nb][q]));
                    }
                }
                const unsigned long long* mine = P.recv[P.rank] + base;
                bool arrived = true;
#pragma unroll
                for (int nb = 0; nb < NB; ++nb)
#pragma unroll
                  for (int q = 0; q < 4; ++q) {
                    const int bb = nb * 8 + 2 * t + (q & 1);
                    const int grow = row * kTileRows + g + 8 * (q >> 1);
                    if (bb < B && grow < N) {
                      const unsigned long long* src = mine + static_cast<size_t>(bb) * P.rows_cap + grow;
                      unsigned long long wv[kMaxPeers];
#pragma unroll
                      for (int r = 0; r < kMaxPeers; ++r)
                        if (r < P.world) wv[r] = ld_word_sys(src + r * slot);
                      float sum = 0.f;
#pragma unroll
                      for (int r = 0; r < kMaxPeers; ++r) {
                        if (r < P.world) {
                          unsigned bits = static_cast<unsigned>(wv[r]);
                          if (static_cast<unsigned>(wv[r] >> 32) != epoch)
                            arrived = wait_word_sys(src + r * slot, epoch, &bits) && arrived;
                          sum += __uint_as_float(bits);
                        }
                      }
                      v[nb][q] = sum;
                    }
                  }
                ok = __all_sync(0xFFFFFFFFu, arrived) && ok;
              }
#pragma unroll
              for (int nb = 0; nb < NB; ++nb)
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  const int bb = nb * 8 + 2 * t + (q & 1);
                  const int grow = row * kTileRows + g + 8 * (q >> 1);
                  if (bb < B && grow < N && ok) y[static_cast<size_t>(bb) * ldy + grow] = v[nb][q];
                }
            }
            row = tr + 1;
            seg_first = i + 1;
          }
        }
      }
      // ---- every consumer warp of the CTA is done with op j (every one
      // reaches this barrier: all their waits are bounded); one thread then
      // publishes the CTA's completion, its fence covering the warps' writes
      named_barrier(1, C * 32);
      if (warp == 0 && lane == 0) {
        __threadfence();
        atomicAdd(p.done + j, 1u);
      }
    }
    // A warp that gave up (a timed-out wait) stopped issuing; its loads still
    // in flight land in this CTA's shared memory, so it waits for them
    // (bounded) before the CTA may exit. On the normal path none are left.
    for (; consumed < issued; ++consumed)
      mbar_wait(&my_full[consumed % D], (consumed / D) & 1u);
  }

  // ---- exit: the last CTA bumps the generation for the next launch
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(p.gen + 1, 1u) == gridDim.x - 1) {
      p.gen[1] = 0u;
      if (p.n_ar > 0) atomicAdd(reinterpret_cast<unsigned*>(p.peers.epoch), static_cast<unsigned>(p.n_ar));
      __threadfence();
      atomicAdd(p.gen, 1u);
    }
  }
}

size_t chain_smem_bytes(bool raw, int consumers, int x_bytes, int batch) {
  const size_t nb = batch <= 8 ? 1 : 2;
  size_t b = 1024;  // alignment slack
  b += static_cast<size_t>(consumers) * kChainSlots * (raw ? kChainSlotRaw : kChainSlotSe12);
  if (!raw) b += static_cast<size_t>(consumers) * kChainSlots * 64;
  b += (static_cast<size_t>(x_bytes) + 15) & ~static_cast<size_t>(15);
  b += static_cast<size_t>(consumers) * 2 * 16 * 8 * nb * 4;               // warps' shares of shared rows
  b += static_cast<size_t>(consumers) * kChainSlots * 8 + 16 + 8;          // barriers, op counters
  b += static_cast<size_t>(consumers) * 2 * 4;                             // row counters
  return b;
}

cudaError_t launch_chain(bool raw, const ChainParams& p, int grid, size_t smem, cudaStream_t stream) {
  using Kernel = void (*)(const ChainParams);
  const Kernel kernel = raw ? (p.batch <= 8 ? chain_kernel<1, true> : chain_kernel<2, true>)
                            : (p.batch <= 8 ? chain_kernel<1, false> : chain_kernel<2, false>);
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3((p.consumers + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  // every CTA waits on the others' progress: all must be resident at once
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, p);
}

}  // namespace se12
