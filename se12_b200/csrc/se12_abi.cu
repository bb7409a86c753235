// C-ABI layer of libse12_b200.so: argument validation, TMA descriptor
// encoding, the fixed launch table, and error reporting. See include/se12.h.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include <cudaTypedefs.h>

#include "../../include/se12.h"
#include "se12_internal.h"

struct se12_matrix {
  se12::MatrixView view;
  alignas(64) CUtensorMap sm_map;
  alignas(64) CUtensorMap ec_map;
  int device;
  int sm_count;
};

namespace {

thread_local std::string g_last_error;

int fail(int status, const std::string& message) {
  g_last_error = message;
  return status;
}

// A CUDA call of this library failed: report it and take it out of the
// thread's last-error state, so that the next call (whose launch checks
// cudaGetLastError) is not blamed for it. A sticky error (a lost context)
// stays, as CUDA keeps it.
int cuda_fail(cudaError_t err, const char* what) {
  (void)cudaGetLastError();
  return fail(SE12_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(err));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

PFN_cuMemGetAddressRange_v3020 address_range_query() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  });
  return fn;
}

int encode_map(CUtensorMap* map, CUtensorMapDataType type, int rank, const void* base, const cuuint64_t* dims,
               const cuuint64_t* strides, const cuuint32_t* box) {
  auto fn = tensor_map_encoder();
  if (!fn) return fail(SE12_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint32_t estride[3] = {1, 1, 1};
  CUresult r = fn(map, type, rank, const_cast<void*>(base), dims, strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SE12_ERR_CUDA, "cuTensorMapEncodeTiled failed with code " + std::to_string(int(r)));
  return SE12_OK;
}

// sm stream as [16T rows][2 halves][128 B] (one box = 4 tiles, both halves);
// ec stream as [16T rows][128 B] (one box = 4 tiles).
int encode_se12_maps(se12_matrix* m) {
  const cuuint64_t rows16 = static_cast<cuuint64_t>(m->view.tiles) * SE12_TILE_ROWS;
  const cuuint32_t box_rows = se12::kSe12BoxTiles * SE12_TILE_ROWS;
  const cuuint64_t sm_dims[3] = {128, 2, rows16};
  const cuuint64_t sm_strides[2] = {128, 256};
  const cuuint32_t sm_box[3] = {128, 2, box_rows};
  int st = encode_map(&m->sm_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, m->view.sm, sm_dims, sm_strides, sm_box);
  if (st != SE12_OK) return st;
  const cuuint64_t ec_dims[2] = {128, rows16};
  const cuuint64_t ec_strides[1] = {128};
  const cuuint32_t ec_box[2] = {128, box_rows};
  return encode_map(&m->ec_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, m->view.ec, ec_dims, ec_strides, ec_box);
}

// Dense W [rows, ldw]: as [rows][cols/64][64] with one box per 16x256 tile
// when cols % 64 == 0, else [rows][cols] with four 16x64 boxes per tile.
int encode_raw_map(CUtensorMap* map, const uint16_t* w, int rows, int cols, int ldw, int* raw_3d) {
  if (cols % 64 == 0) {
    const cuuint64_t dims[3] = {64, static_cast<cuuint64_t>(cols / 64), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[2] = {128, static_cast<cuuint64_t>(ldw) * 2};
    const cuuint32_t box[3] = {64, 4, 16};
    *raw_3d = 1;
    return encode_map(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, w, dims, strides, box);
  }
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldw) * 2};
  const cuuint32_t box[2] = {64, 16};
  *raw_3d = 0;
  return encode_map(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, dims, strides, box);
}

int current_device_info(int* device, int* sm_count) {
  cudaError_t err = cudaGetDevice(device);
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetDevice");
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, *device);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, *device);
  if (major != 10 || minor != 0)
    return fail(SE12_ERR_UNSUPPORTED_DEVICE, "libse12_b200 is built for sm_100a; device has compute capability " +
                                                 std::to_string(major) + "." + std::to_string(minor));
  err = cudaDeviceGetAttribute(sm_count, cudaDevAttrMultiProcessorCount, *device);
  if (err != cudaSuccess) return cuda_fail(err, "cudaDeviceGetAttribute");
  return SE12_OK;
}

int tiles_of(int rows, int cols) {
  return ((rows + SE12_TILE_ROWS - 1) / SE12_TILE_ROWS) * ((cols + SE12_TILE_COLS - 1) / SE12_TILE_COLS);
}

// ------------------------------------------------------------------ launch table
//
// The fixed launch table that replaces the reference's run-time tuner
// (lws.tune, src/lws/tune.py:34-57). The tile is fixed by the format
// (16x256); what varies is the stage (4 or 8 tiles), the pipeline depth,
// whether x is resident, the grid and how tiles map to CTAs.
//  * Shared memory: the first candidate (below) that lets two CTAs share an
//    SM, for each stage size; only if no candidate does, one CTA per SM.
//    8-tile stages need x resident.
//  * Work split: row mode (whole tile rows per CTA, no cross-CTA fixup) or
//    stream-K (equal runs of stages, split rows finished across CTAs).
//  * Among these, the smallest critical path of the longest CTA: stages x
//    stage time + the stream-K fixup. In units of a 4-tile stage's overhead-
//    inclusive half-tile time: a 4-tile stage (two CTAs per SM) costs 1.65,
//    an 8-tile stage 2.0 (each warp does a whole tile, decoding it group by
//    group); x 0.95 when one CTA has the SM to itself, x 1.6 for two CTAs
//    per SM at batch 9..16 (their build spills, the one-CTA build does
//    not), x 1.5 when x is staged; a fixup 3.0 (a round trip through L2 on
//    a loaded GPU). The
//    wide layout (SE12, x resident, one CTA per SM with kWideGroups 4-tile
//    stages in work at once, row mode only) costs 3.0 per CTA (its longer
//    fill and drain) + 0.48 per 4-tile stage: it streams a little faster and
//    starts slower, so it wins on large matrices only. Fitted
//    to stacked timings of every choice on Gemma-2 2B/9B/27B shapes at batch
//    1, 4 and 16.
struct LaunchConfig {
  int grid;
  int stages;
  int nblocks;
  int x_resident;
  int row_mode;
  int full_tiles;
  int wide;
  size_t smem;
};

struct MemoryChoice {
  int x_resident, stages, per_sm;  // per_sm = 0: none fits
};

// 8-tile stages only with x resident: their staged x (twice that of a
// 4-tile stage) leaves room for two stages only and measured slower.
MemoryChoice choose_memory(bool raw, bool full, int batch, int cols) {
  // (x resident?, stages) in order of preference
  static const int kOrder[][2] = {{1, 4}, {1, 3}, {0, 4}, {0, 3}, {1, 2}, {0, 2}};
  for (const size_t limit : {se12::kCoResidentSmem, se12::kMaxSmemPerCta}) {
    // 8-tile stages in one CTA per SM: two stages, which measured faster
    // than three or four at batch 1-4 (the 2B down projection at batch 4
    // 12.5 against 13.1 us; q/k/v, gate/up and the 9B shapes by 1-5 %)
    if (full && limit == se12::kMaxSmemPerCta) {
      if (se12::gemv_smem_bytes(raw, true, true, 2, batch, cols) + 1024 <= limit) return {1, 2, 1};
      break;
    }
    for (const auto& cand : kOrder) {
      if (full && !cand[0]) continue;
      if (se12::gemv_smem_bytes(raw, full, cand[0] != 0, cand[1], batch, cols) <= limit)
        return {cand[0], cand[1], limit == se12::kCoResidentSmem ? 2 : 1};
    }
  }
  return {0, 0, 0};
}

// The wide layout (one CTA per SM, kWideGroups stages in work at once):
// x resident and a pipeline of kWideGroups + 2 stages, so that two stages
// are in flight, if it fits (with 1 KB to spare for the kernel's static
// shared memory). Deeper pipelines measured slower with 4 groups (the 2B
// lm_head 195.0 / 195.3 / 195.8 us at 6 / 7 / 8 stages; down 12.4 / 12.8 /
// 13.0 us; gate/up at batch 4 20.0 / 20.3 / 20.5 us).
MemoryChoice choose_memory_wide(int batch, int cols) {
  if (batch > 8) return {0, 0, 0};  // one block of 8 batch columns (two spill at 96 registers)
  const int stages = se12::kWideGroups + 2;
  if (se12::gemv_smem_bytes(false, false, true, stages, batch, cols, true) + 1024 <= se12::kMaxSmemPerCta)
    return {1, stages, 1};
  return {0, 0, 0};
}

LaunchConfig choose_config(bool raw, int tiles, int cols, int batch, int sm_count, bool allow_wide = true) {
  const MemoryChoice mem4 = choose_memory(raw, false, batch, cols);
  const MemoryChoice mem8 = raw ? MemoryChoice{0, 0, 0} : choose_memory(raw, true, batch, cols);
  const int tile_cols = (cols + SE12_TILE_COLS - 1) / SE12_TILE_COLS;
  const int tile_rows = tiles / tile_cols;
  constexpr double kStageCost4 = 1.65;  // a 4-tile stage, two CTAs per SM, x resident
  constexpr double kStageCost8 = 2.0;   // an 8-tile stage
  constexpr double kAloneFactor = 0.95;
  constexpr double kStagedXFactor = 1.5;
  // batch 9..16 with two CTAs per SM: that build (96 registers) spills its
  // two-block accumulators, the one-CTA build does not
  constexpr double kSharedTwoBlocks = 1.6;
  constexpr double kFixup = 3.0;
  constexpr double kWideFixed = 3.0;   // the wide layout: a longer pipeline fill and drain per CTA,
  constexpr double kWideStage = 0.48;  // then a 4-tile stage (kWideGroups in work at once, one CTA per SM)
  LaunchConfig best{};
  double best_cost = 0;
  for (const bool full : {false, true}) {
    const MemoryChoice& mem = full ? mem8 : mem4;
    if (!mem.per_sm) continue;
    const int stage = se12::stage_tiles(full);
    const double stage_cost = (full ? kStageCost8 : kStageCost4) *
                              (mem.per_sm == 1 ? kAloneFactor : (batch > 8 ? kSharedTwoBlocks : 1.0)) *
                              (mem.x_resident ? 1.0 : kStagedXFactor);
    const int slots = mem.per_sm * sm_count;
    const int units = (tiles + stage - 1) / stage;
    const int grid_sk = std::max(1, std::min(units, slots));
    const int grid_rows = std::max(1, std::min(tile_rows, slots));
    const int stages_sk = (units + grid_sk - 1) / grid_sk;
    const int rows_per_cta = (tile_rows + grid_rows - 1) / grid_rows;
    const int stages_rows = (rows_per_cta * tile_cols + stage - 1) / stage;
    for (const int row_mode : {1, 0}) {
      const double cost = row_mode ? stages_rows * stage_cost : stages_sk * stage_cost + kFixup;
      if (best.stages && cost >= best_cost) continue;
      best_cost = cost;
      best.full_tiles = full ? 1 : 0;
      best.x_resident = mem.x_resident;
      best.stages = mem.stages;
      best.row_mode = row_mode;
      best.grid = row_mode ? grid_rows : grid_sk;
    }
  }
  // Every tile row in one wave of one CTA per SM, and 8-tile stages that
  // hold one CTA per SM: those run faster than the wide layout (the 2B down
  // projection, 144 rows of 36 tiles: 12.16 against 12.37 us at batch 1,
  // 12.23 against 12.52 at batch 2)
  const bool one_wave_full = !raw && mem8.per_sm == 1 && tile_rows <= sm_count;
  const MemoryChoice memw =
      (raw || !allow_wide || one_wave_full) ? MemoryChoice{0, 0, 0} : choose_memory_wide(batch, cols);
  if (memw.per_sm) {
    // row mode only: with the fixup, stream-K in the wide layout never
    // beats stream-K in the others (finer grained, two CTAs per SM)
    const int stage = se12::stage_tiles(false);
    const int grid_rows = std::max(1, std::min(tile_rows, sm_count));
    const int rows_per_cta = (tile_rows + grid_rows - 1) / grid_rows;
    const int stages_rows = (rows_per_cta * tile_cols + stage - 1) / stage;
    const double cost = kWideFixed + stages_rows * kWideStage;
    if (!best.stages || cost < best_cost) {
      best_cost = cost;
      best.full_tiles = 0;
      best.wide = 1;
      best.x_resident = 1;
      best.stages = memw.stages;
      best.row_mode = 1;
      best.grid = grid_rows;
    }
  }
  if (!best.stages) {  // not reached for batch <= 16: 4-tile stages with staged x, 2 stages, fit one CTA per SM
    best.stages = 2;
    best.grid = std::max(1, std::min((tiles + 3) / 4, sm_count));
  }
  best.nblocks = batch <= 8 ? 1 : 2;
  best.smem = se12::gemv_smem_bytes(raw, best.full_tiles != 0, best.x_resident != 0, best.stages, batch, cols,
                                    best.wide != 0);
  return best;
}

// Workspace layout, identical for every matrix so that all calls on one
// stream can share one workspace: [partials][flags]. The partials region
// has a fixed size (the largest grid and batch: 2 CTAs per SM, 2 slots of
// 16 rows x 16 batch columns each); the flags (one int per CTA, "partial
// published", zero between calls) follow it.
size_t partials_region_bytes(int sm_count) { return static_cast<size_t>(2 * sm_count) * 2 * 16 * 16 * 4; }

size_t workspace_bytes_for(int /*tile_rows*/, int sm_count) {
  return partials_region_bytes(sm_count) + (static_cast<size_t>(2 * sm_count) * 4 + 255) / 256 * 256;
}

}  // namespace

extern "C" {

int se12_abi_version(void) { return 1; }

const char* se12_last_error(void) { return g_last_error.c_str(); }

const char* se12_status_string(int status) {
  switch (status) {
    case SE12_OK: return "ok";
    case SE12_ERR_INVALID_ARGUMENT: return "invalid argument";
    case SE12_ERR_UNSUPPORTED_FORMAT: return "unsupported SE12 format";
    case SE12_ERR_MISALIGNED: return "misaligned pointer or leading dimension";
    case SE12_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
    case SE12_ERR_CUDA: return "CUDA error";
    case SE12_ERR_UNSUPPORTED_DEVICE: return "unsupported device (needs sm_100)";
    case SE12_ERR_DEVICE_FAULT: return "a kernel reported an error";
    default: return "unknown status";
  }
}

size_t se12_escape_pos_bytes(int rows, int cols) {
  return static_cast<size_t>(tiles_of(rows, cols)) * SE12_ESCAPE_BUDGET * sizeof(uint16_t);
}

size_t se12_fallback_index_bytes(int rows, int cols) {
  return static_cast<size_t>((tiles_of(rows, cols) + 3) & ~3) * sizeof(int32_t);
}

int se12_matrix_create(const se12_streams* s, se12_matrix** out) {
  if (!s) return fail(SE12_ERR_INVALID_ARGUMENT, "null argument");
  return se12_matrix_create_segmented(s, 1, &s->rows, s->codebook, out);
}

int se12_matrix_create_segmented(const se12_streams* s, int segments, const int32_t* segment_rows,
                                 const uint8_t* codebooks, se12_matrix** out) {
  if (!s || !out || !segment_rows || !codebooks) return fail(SE12_ERR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  if (segments < 1 || segments > SE12_MAX_SEGMENTS)
    return fail(SE12_ERR_INVALID_ARGUMENT, "segments must be in 1.." + std::to_string(SE12_MAX_SEGMENTS));
  long long total_rows = 0;
  for (int i = 0; i < segments; ++i) {
    if (segment_rows[i] <= 0) return fail(SE12_ERR_INVALID_ARGUMENT, "segment rows must be positive");
    if (i + 1 < segments && segment_rows[i] % SE12_TILE_ROWS != 0)
      return fail(SE12_ERR_INVALID_ARGUMENT, "every segment but the last needs a multiple of 16 rows");
    total_rows += segment_rows[i];
  }
  if (total_rows != s->rows)
    return fail(SE12_ERR_INVALID_ARGUMENT, "segment rows sum to " + std::to_string(total_rows) + ", streams have " +
                                               std::to_string(s->rows) + " rows");
  if (s->tile_rows != SE12_TILE_ROWS || s->tile_cols != SE12_TILE_COLS || s->escape_budget != SE12_ESCAPE_BUDGET)
    return fail(SE12_ERR_UNSUPPORTED_FORMAT, "tile shape must be 16x256 with an escape budget of 16, got " +
                                                 std::to_string(s->tile_rows) + "x" + std::to_string(s->tile_cols) +
                                                 " / " + std::to_string(s->escape_budget));
  if (s->format_version != SE12_FORMAT_VERSION)
    return fail(SE12_ERR_UNSUPPORTED_FORMAT,
                "found format version " + std::to_string(s->format_version) + ", supported: 1");
  if (s->rows <= 0 || s->cols <= 0) return fail(SE12_ERR_INVALID_ARGUMENT, "rows and cols must be positive");
  if (!s->sm || !s->ec || !s->esc || !s->fallback_bitmap || !s->escape_pos || !s->fallback_index)
    return fail(SE12_ERR_INVALID_ARGUMENT, "null stream pointer");
  if (!aligned16(s->sm) || !aligned16(s->ec) || !aligned16(s->esc) || !aligned16(s->escape_pos) ||
      !aligned16(s->fallback_index) || (s->fallback_raw && !aligned16(s->fallback_raw)))
    return fail(SE12_ERR_MISALIGNED, "SE12 streams must be 16-byte aligned");
  int device = 0, sm_count = 0;
  int st = current_device_info(&device, &sm_count);
  if (st != SE12_OK) return st;

  se12_matrix* m = new se12_matrix();
  se12::MatrixView& v = m->view;
  v.sm = s->sm;
  v.ec = s->ec;
  v.esc = s->esc;
  v.bitmap = s->fallback_bitmap;
  v.fallback_raw = reinterpret_cast<const uint16_t*>(s->fallback_raw);
  v.escape_pos = s->escape_pos;
  v.fallback_index = s->fallback_index;
  v.rows = s->rows;
  v.cols = s->cols;
  v.tile_rows = (s->rows + SE12_TILE_ROWS - 1) / SE12_TILE_ROWS;
  v.tile_cols = (s->cols + SE12_TILE_COLS - 1) / SE12_TILE_COLS;
  v.tiles = v.tile_rows * v.tile_cols;
  std::memset(v.codebooks, 0, sizeof(v.codebooks));
  v.segments = segments;
  int end = 0;
  for (int i = 0; i < se12::kMaxSegments; ++i) {
    if (i < segments) {
      end += (segment_rows[i] + SE12_TILE_ROWS - 1) / SE12_TILE_ROWS;
      std::memcpy(v.codebooks[i], codebooks + i * SE12_CODEBOOK_SIZE, SE12_CODEBOOK_SIZE);
    }
    v.seg_end[i] = (i < segments - 1) ? end : INT32_MAX;
  }
  m->device = device;
  m->sm_count = sm_count;
  st = encode_se12_maps(m);
  if (st != SE12_OK) {
    delete m;
    return st;
  }
  *out = m;
  return SE12_OK;
}

int se12_matrix_prepare(const se12_matrix* m, void* stream) {
  if (!m) return fail(SE12_ERR_INVALID_ARGUMENT, "null matrix");
  cudaError_t err = se12::launch_prepare(m->view, const_cast<uint16_t*>(m->view.escape_pos),
                                         const_cast<int32_t*>(m->view.fallback_index),
                                         static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "se12_matrix_prepare launch");
  return SE12_OK;
}

void se12_matrix_destroy(se12_matrix* m) { delete m; }

size_t se12_gemv_workspace_bytes(const se12_matrix* m, int batch) {
  if (!m || batch < 1 || batch > SE12_MAX_BATCH) return 0;
  return workspace_bytes_for(m->view.tile_rows, m->sm_count);
}

int se12_workspace_clear(void* workspace, size_t bytes, void* stream) {
  if (!workspace && bytes) return fail(SE12_ERR_INVALID_ARGUMENT, "null workspace");
  cudaError_t err = cudaMemsetAsync(workspace, 0, bytes, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "cudaMemsetAsync");
  return SE12_OK;
}

static int check_gemv_io(int rows, int cols, const uint16_t* x, int batch, int ldx, const float* y, int ldy) {
  if (batch < 1 || batch > SE12_MAX_BATCH)
    return fail(SE12_ERR_INVALID_ARGUMENT, "batch must be in 1..16, got " + std::to_string(batch));
  if (!x || !y) return fail(SE12_ERR_INVALID_ARGUMENT, "null x or y");
  if (ldx < (cols + 7) / 8 * 8 || ldy < rows)
    return fail(SE12_ERR_INVALID_ARGUMENT, "ldx < cols rounded up to 8, or ldy < rows");
  if (!aligned16(x) || (ldx % 8) != 0)
    return fail(SE12_ERR_MISALIGNED, "x must be 16-byte aligned with ldx a multiple of 8");
  return SE12_OK;
}

static void fill_launch_config(const LaunchConfig& c, se12_launch_config* out) {
  out->grid = c.grid;
  out->threads = se12::gemv_threads(c.wide != 0);
  out->smem_bytes = static_cast<int>(c.smem);
  out->ctas_per_sm = (c.smem <= se12::kCoResidentSmem && !c.wide) ? 2 : 1;
  out->stage_tiles = se12::stage_tiles(c.full_tiles != 0);
  out->stages = c.stages;
  out->x_resident = c.x_resident;
  out->row_mode = c.row_mode;
  out->wide = c.wide;
}

int se12_gemv_launch_config(const se12_matrix* m, int batch, se12_launch_config* out) {
  if (!m || !out) return fail(SE12_ERR_INVALID_ARGUMENT, "null argument");
  if (batch < 1 || batch > SE12_MAX_BATCH)
    return fail(SE12_ERR_INVALID_ARGUMENT, "batch must be in 1.." + std::to_string(SE12_MAX_BATCH));
  fill_launch_config(choose_config(false, m->view.tiles, m->view.cols, batch, m->sm_count), out);
  return SE12_OK;
}

int se12_gemv_plan(int rows, int cols, int batch, int sm_count, se12_launch_config* out) {
  if (!out) return fail(SE12_ERR_INVALID_ARGUMENT, "null argument");
  if (rows <= 0 || cols <= 0) return fail(SE12_ERR_INVALID_ARGUMENT, "rows and cols must be positive");
  if (batch < 1 || batch > SE12_MAX_BATCH)
    return fail(SE12_ERR_INVALID_ARGUMENT, "batch must be in 1.." + std::to_string(SE12_MAX_BATCH));
  if (sm_count < 1 || sm_count > 1024) return fail(SE12_ERR_INVALID_ARGUMENT, "sm_count must be in 1..1024");
  fill_launch_config(choose_config(false, tiles_of(rows, cols), cols, batch, sm_count), out);
  return SE12_OK;
}

int se12_gemv(const se12_matrix* m, const uint16_t* x, int batch, int ldx, float* y, int ldy, void* workspace,
              size_t workspace_bytes, void* stream) {
  if (!m) return fail(SE12_ERR_INVALID_ARGUMENT, "null matrix");
  int st = check_gemv_io(m->view.rows, m->view.cols, x, batch, ldx, y, ldy);
  if (st != SE12_OK) return st;
  const LaunchConfig c = choose_config(false, m->view.tiles, m->view.cols, batch, m->sm_count);
  const size_t need = workspace_bytes_for(m->view.tile_rows, m->sm_count);
  if (!workspace || workspace_bytes < need)
    return fail(SE12_ERR_WORKSPACE_TOO_SMALL, "workspace needs " + std::to_string(need) + " bytes");
  se12::GemvArgs a{};
  a.m = m->view;
  a.x = x;
  a.ldx = ldx;
  a.batch = batch;
  a.y = y;
  a.ldy = ldy;
  a.partials = static_cast<float*>(workspace);
  a.counters = reinterpret_cast<int*>(static_cast<char*>(workspace) + partials_region_bytes(m->sm_count));
  a.grid = c.grid;
  a.stages = c.stages;
  a.x_resident = c.x_resident;
  a.row_mode = c.row_mode;
  a.full_tiles = c.full_tiles;
  a.wide = c.wide;
  cudaError_t err = se12::launch_gemv(false, m->sm_map, m->ec_map, a, c.nblocks, c.smem,
                                      static_cast<cudaStream_t>(stream), true);
  if (err != cudaSuccess) return cuda_fail(err, "se12_gemv launch");
  return SE12_OK;
}

int bf16_gemv_plan(int rows, int cols, int batch, int sm_count, se12_launch_config* out) {
  if (!out || rows <= 0 || cols <= 0 || batch < 1 || batch > SE12_MAX_BATCH || sm_count <= 0)
    return fail(SE12_ERR_INVALID_ARGUMENT, "bad shape, batch or SM count");
  fill_launch_config(choose_config(true, tiles_of(rows, cols), cols, batch, sm_count), out);
  return SE12_OK;
}

int se12_gemv_order_matched(const se12_matrix* m, const uint16_t* x, int batch, int ldx, float* y, int ldy,
                            void* workspace, size_t workspace_bytes, void* stream) {
  if (!m) return fail(SE12_ERR_INVALID_ARGUMENT, "null matrix");
  int st = check_gemv_io(m->view.rows, m->view.cols, x, batch, ldx, y, ldy);
  if (st != SE12_OK) return st;
  // bf16_gemv's configuration for this shape (4-tile stages, never the wide
  // layout), with the SE12 kernel's own shared-memory size for it
  LaunchConfig c = choose_config(true, m->view.tiles, m->view.cols, batch, m->sm_count);
  c.smem = se12::gemv_smem_bytes(false, false, c.x_resident != 0, c.stages, batch, m->view.cols, false);
  if (c.smem > se12::kMaxSmemPerCta)
    return fail(SE12_ERR_UNSUPPORTED_DEVICE, "the dense kernel's configuration does not fit the SE12 kernel");
  const size_t need = workspace_bytes_for(m->view.tile_rows, m->sm_count);
  if (!workspace || workspace_bytes < need)
    return fail(SE12_ERR_WORKSPACE_TOO_SMALL, "workspace needs " + std::to_string(need) + " bytes");
  se12::GemvArgs a{};
  a.m = m->view;
  a.x = x;
  a.ldx = ldx;
  a.batch = batch;
  a.y = y;
  a.ldy = ldy;
  a.partials = static_cast<float*>(workspace);
  a.counters = reinterpret_cast<int*>(static_cast<char*>(workspace) + partials_region_bytes(m->sm_count));
  a.grid = c.grid;
  a.stages = c.stages;
  a.x_resident = c.x_resident;
  a.row_mode = c.row_mode;
  a.full_tiles = 0;
  a.wide = 0;
  cudaError_t err = se12::launch_gemv(false, m->sm_map, m->ec_map, a, c.nblocks, c.smem,
                                      static_cast<cudaStream_t>(stream), true);
  if (err != cudaSuccess) return cuda_fail(err, "se12_gemv_order_matched launch");
  return SE12_OK;
}

int se12_ipc_handle(const void* dev_ptr, uint8_t* handle_out, uint64_t* offset_out) {
  if (!dev_ptr || !handle_out || !offset_out) return fail(SE12_ERR_INVALID_ARGUMENT, "null argument");
  auto range = address_range_query();
  if (!range) return fail(SE12_ERR_CUDA, "cuMemGetAddressRange is not available");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
    return fail(SE12_ERR_INVALID_ARGUMENT, "not a device allocation");
  cudaIpcMemHandle_t h;
  cudaError_t err = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (err != cudaSuccess) return cuda_fail(err, "cudaIpcGetMemHandle");
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = reinterpret_cast<uint64_t>(dev_ptr) - static_cast<uint64_t>(base);
  return SE12_OK;
}

int se12_ipc_open(const uint8_t* handle, uint64_t offset, void** dev_ptr_out, void** mapping_out) {
  if (!handle || !dev_ptr_out || !mapping_out) return fail(SE12_ERR_INVALID_ARGUMENT, "null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  cudaError_t err = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (err != cudaSuccess) return cuda_fail(err, "cudaIpcOpenMemHandle");
  *mapping_out = p;
  *dev_ptr_out = static_cast<char*>(p) + offset;
  return SE12_OK;
}

int se12_ipc_close(void* mapping) {
  if (!mapping) return SE12_OK;
  cudaError_t err = cudaIpcCloseMemHandle(mapping);
  if (err != cudaSuccess) return cuda_fail(err, "cudaIpcCloseMemHandle");
  return SE12_OK;
}

size_t se12_peer_recv_bytes(int world, int rows_cap) {
  if (world < 1 || world > SE12_MAX_PEERS || rows_cap < 1) return 0;
  return static_cast<size_t>(2) * world * 16 * rows_cap * sizeof(uint64_t);
}

}  // extern "C"

static int gemv_peers(const se12_matrix* m, const uint16_t* x, int batch, int ldx, float* y, int ldy, void* workspace,
                      size_t workspace_bytes, const se12_peer_group* g, void* stream, int gather, int row0, int rows_full) {
  if (!m || !g) return fail(SE12_ERR_INVALID_ARGUMENT, "null matrix or peer group");
  if (g->world < 2 || g->world > SE12_MAX_PEERS || g->rank < 0 || g->rank >= g->world)
    return fail(SE12_ERR_INVALID_ARGUMENT, "peer group needs 2.." + std::to_string(SE12_MAX_PEERS) +
                                               " ranks and 0 <= rank < world");
  if (!gather && m->view.rows > g->rows_cap)
    return fail(SE12_ERR_INVALID_ARGUMENT, "matrix has " + std::to_string(m->view.rows) +
                                               " rows, the peer buffers hold " + std::to_string(g->rows_cap));
  if (gather && (row0 < 0 || rows_full < row0 + m->view.rows ||
                 static_cast<long long>(rows_full) > static_cast<long long>(g->world) * g->rows_cap))
    return fail(SE12_ERR_INVALID_ARGUMENT, "gathered rows: need 0 <= row0, row0 + matrix rows <= rows_full <= world x "
                                           "rows_cap (" + std::to_string(g->world) + " x " + std::to_string(g->rows_cap) + ")");
  if (!g->epoch) return fail(SE12_ERR_INVALID_ARGUMENT, "null epoch counter");
  for (int r = 0; r < g->world; ++r) {
    if (!g->recv[r]) return fail(SE12_ERR_INVALID_ARGUMENT, "null peer buffer");
    if (!aligned16(g->recv[r]))
      return fail(SE12_ERR_MISALIGNED, "peer buffers must be 16-byte aligned");
  }
  int st = check_gemv_io(gather ? rows_full : m->view.rows, m->view.cols, x, batch, ldx, y, ldy);
  if (st != SE12_OK) return st;
  const LaunchConfig c = choose_config(false, m->view.tiles, m->view.cols, batch, m->sm_count, false);
  const size_t need = workspace_bytes_for(m->view.tile_rows, m->sm_count);
  if (!workspace || workspace_bytes < need)
    return fail(SE12_ERR_WORKSPACE_TOO_SMALL, "workspace needs " + std::to_string(need) + " bytes");
  se12::GemvArgs a{};
  a.m = m->view;
  a.x = x;
  a.ldx = ldx;
  a.batch = batch;
  a.y = y;
  a.ldy = ldy;
  a.partials = static_cast<float*>(workspace);
  a.counters = reinterpret_cast<int*>(static_cast<char*>(workspace) + partials_region_bytes(m->sm_count));
  a.grid = c.grid;
  a.stages = c.stages;
  a.x_resident = c.x_resident;
  a.row_mode = c.row_mode;
  a.full_tiles = c.full_tiles;
  a.wide = c.wide;
  a.peers.world = g->world;
  a.peers.rank = g->rank;
  a.peers.rows_cap = g->rows_cap;
  for (int r = 0; r < g->world; ++r) {
    a.peers.recv[r] = static_cast<unsigned long long*>(g->recv[r]);
  }
  a.peers.epoch = g->epoch;
  a.peers.gather = gather;
  a.peers.row0 = row0;
  a.peers.rows_full = rows_full;
  cudaError_t err = se12::launch_gemv(false, m->sm_map, m->ec_map, a, c.nblocks, c.smem,
                                      static_cast<cudaStream_t>(stream), true);
  if (err != cudaSuccess) return cuda_fail(err, gather ? "se12_gemv_allgather launch" : "se12_gemv_allreduce launch");
  return SE12_OK;
}

extern "C" {

int se12_gemv_allreduce(const se12_matrix* m, const uint16_t* x, int batch, int ldx, float* y, int ldy, void* workspace,
                        size_t workspace_bytes, const se12_peer_group* g, void* stream) {
  return gemv_peers(m, x, batch, ldx, y, ldy, workspace, workspace_bytes, g, stream, 0, 0, 0);
}

int se12_gemv_allgather(const se12_matrix* m, const uint16_t* x, int batch, int ldx, float* y, int ldy, int row0,
                        int rows_full, void* workspace, size_t workspace_bytes, const se12_peer_group* g, void* stream) {
  return gemv_peers(m, x, batch, ldx, y, ldy, workspace, workspace_bytes, g, stream, 1, row0, rows_full);
}

}  // extern "C"

// ------------------------------------------------------------------ no-allocation GEMV
// Scratch of se12_gemv_noalloc, for callers that cannot allocate device
// memory: the stream-K partial rows of up to kNoAllocMaxGrid CTAs, then one
// flag per CTA. It is part of the library's device image, so every GPU that
// loads the library holds these 644 KiB until the process exits.
namespace {
constexpr int kNoAllocMaxGrid = 320;
constexpr size_t kNoAllocPartialsBytes = static_cast<size_t>(kNoAllocMaxGrid) * 2 * 16 * 16 * sizeof(float);
constexpr size_t kNoAllocScratchBytes = kNoAllocPartialsBytes + 4096;  // + kNoAllocMaxGrid flags, padded
constexpr int kNoAllocMaxDevices = 64;

std::mutex g_noalloc_mutex;
void* g_noalloc_scratch_ptr[kNoAllocMaxDevices] = {};
}  // namespace

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the scratch on `device` (the current device). The first
// call on a device looks it up with cudaGetSymbolAddress; later calls reuse it.
static int noalloc_scratch(int device, void** out) {
  if (device < 0 || device >= kNoAllocMaxDevices)
    return fail(SE12_ERR_UNSUPPORTED_DEVICE, "se12_gemv_noalloc supports device ordinals below 64");
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_scratch_ptr[device]) {
    void* ptr = nullptr;
    cudaError_t err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (err != cudaSuccess) return cuda_fail(err, "cudaGetSymbolAddress of the se12_gemv_noalloc scratch");
    g_noalloc_scratch_ptr[device] = ptr;
  }
  *out = g_noalloc_scratch_ptr[device];
  return SE12_OK;
}

extern "C" {

int se12_gemv_noalloc(const se12_matrix* m, const uint16_t* x, int batch, int ldx, float* y, int ldy, void* stream) {
  if (!m) return fail(SE12_ERR_INVALID_ARGUMENT, "null matrix");
  int st = check_gemv_io(m->view.rows, m->view.cols, x, batch, ldx, y, ldy);
  if (st != SE12_OK) return st;
  int device = -1;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetDevice");
  if (device != m->device)
    return fail(SE12_ERR_INVALID_ARGUMENT, "se12_gemv_noalloc: the current device (" + std::to_string(device) +
                                               ") is not the matrix's device (" + std::to_string(m->device) + ")");
  const LaunchConfig c = choose_config(false, m->view.tiles, m->view.cols, batch, m->sm_count);
  if (c.grid > kNoAllocMaxGrid)
    return fail(SE12_ERR_UNSUPPORTED_DEVICE, "se12_gemv_noalloc supports grids of at most " +
                                                 std::to_string(kNoAllocMaxGrid) + " CTAs, this device needs " +
                                                 std::to_string(c.grid));
  void* scratch = nullptr;
  st = noalloc_scratch(device, &scratch);
  if (st != SE12_OK) return st;
  int* counters = reinterpret_cast<int*>(static_cast<char*>(scratch) + kNoAllocPartialsBytes);
  // The per-CTA flags must start at zero; a completed call leaves them at
  // zero, but clearing them here also recovers from a call that did not
  // complete.
  err = cudaMemsetAsync(counters, 0, static_cast<size_t>(c.grid) * sizeof(int), static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "cudaMemsetAsync of the se12_gemv_noalloc counters");
  se12::GemvArgs a{};
  a.m = m->view;
  a.x = x;
  a.ldx = ldx;
  a.batch = batch;
  a.y = y;
  a.ldy = ldy;
  a.partials = static_cast<float*>(scratch);
  a.counters = counters;
  a.grid = c.grid;
  a.stages = c.stages;
  a.x_resident = c.x_resident;
  a.row_mode = c.row_mode;
  a.full_tiles = c.full_tiles;
  a.wide = c.wide;
  err = se12::launch_gemv(false, m->sm_map, m->ec_map, a, c.nblocks, c.smem, static_cast<cudaStream_t>(stream), false);
  if (err != cudaSuccess) return cuda_fail(err, "se12_gemv_noalloc launch");
  return SE12_OK;
}

int se12_decode(const se12_matrix* m, uint16_t* out, int ldo, void* stream) {
  if (!m || !out) return fail(SE12_ERR_INVALID_ARGUMENT, "null argument");
  if (ldo < m->view.cols) return fail(SE12_ERR_INVALID_ARGUMENT, "ldo < cols");
  cudaError_t err = se12::launch_decode(m->view, out, ldo, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "se12_decode launch");
  return SE12_OK;
}

int se12_decode_rows(const se12_matrix* m, const int32_t* rows, int nrows, uint16_t* out, int ldo, void* stream) {
  if (!m || (nrows > 0 && (!rows || !out))) return fail(SE12_ERR_INVALID_ARGUMENT, "null argument");
  if (nrows < 0 || ldo < m->view.cols) return fail(SE12_ERR_INVALID_ARGUMENT, "nrows < 0 or ldo < cols");
  cudaError_t err = se12::launch_decode_rows(m->view, rows, nrows, out, ldo, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "se12_decode_rows launch");
  return SE12_OK;
}

size_t bf16_gemv_workspace_bytes(int rows, int cols, int batch) {
  if (rows <= 0 || cols <= 0 || batch < 1 || batch > SE12_MAX_BATCH) return 0;
  int device = 0, sm_count = 148;
  if (cudaGetDevice(&device) == cudaSuccess) cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, device);
  return workspace_bytes_for((rows + SE12_TILE_ROWS - 1) / SE12_TILE_ROWS, sm_count);
}

int bf16_gemv(const uint16_t* w, int rows, int cols, int ldw, const uint16_t* x, int batch, int ldx, float* y,
              int ldy, void* workspace, size_t workspace_bytes, void* stream) {
  if (!w) return fail(SE12_ERR_INVALID_ARGUMENT, "null weights");
  if (rows <= 0 || cols <= 0 || ldw < cols) return fail(SE12_ERR_INVALID_ARGUMENT, "bad weight shape");
  if (!aligned16(w) || (ldw % 8) != 0) return fail(SE12_ERR_MISALIGNED, "W must be 16-byte aligned, ldw % 8 == 0");
  int st = check_gemv_io(rows, cols, x, batch, ldx, y, ldy);
  if (st != SE12_OK) return st;
  int device = 0, sm_count = 0;
  st = current_device_info(&device, &sm_count);
  if (st != SE12_OK) return st;
  const int tile_rows = (rows + SE12_TILE_ROWS - 1) / SE12_TILE_ROWS;
  const int tile_cols = (cols + SE12_TILE_COLS - 1) / SE12_TILE_COLS;
  const LaunchConfig c = choose_config(true, tile_rows * tile_cols, cols, batch, sm_count);
  const size_t need = workspace_bytes_for(tile_rows, sm_count);
  if (!workspace || workspace_bytes < need)
    return fail(SE12_ERR_WORKSPACE_TOO_SMALL, "workspace needs " + std::to_string(need) + " bytes");
  alignas(64) CUtensorMap wmap;
  int raw_3d = 0;
  st = encode_raw_map(&wmap, w, rows, cols, ldw, &raw_3d);
  if (st != SE12_OK) return st;
  se12::GemvArgs a{};
  a.raw_3d = raw_3d;
  a.m.rows = rows;
  a.m.cols = cols;
  a.m.tile_rows = tile_rows;
  a.m.tile_cols = tile_cols;
  a.m.tiles = tile_rows * tile_cols;
  a.m.segments = 1;
  for (int i = 0; i < se12::kMaxSegments; ++i) a.m.seg_end[i] = INT32_MAX;
  a.x = x;
  a.ldx = ldx;
  a.batch = batch;
  a.y = y;
  a.ldy = ldy;
  a.partials = static_cast<float*>(workspace);
  a.counters = reinterpret_cast<int*>(static_cast<char*>(workspace) + partials_region_bytes(sm_count));
  a.grid = c.grid;
  a.stages = c.stages;
  a.x_resident = c.x_resident;
  a.row_mode = c.row_mode;
  a.full_tiles = c.full_tiles;
  a.wide = c.wide;
  cudaError_t err = se12::launch_gemv(true, wmap, wmap, a, c.nblocks, c.smem, static_cast<cudaStream_t>(stream), true);
  if (err != cudaSuccess) return cuda_fail(err, "bf16_gemv launch");
  return SE12_OK;
}

int se12_encode_histogram(const uint16_t* w, int rows, int cols, int ldw, uint32_t* counts, void* stream) {
  if (!w || !counts || rows < 0 || cols < 0 || ldw < cols) return fail(SE12_ERR_INVALID_ARGUMENT, "bad arguments");
  cudaError_t err = se12::launch_encode_histogram(w, rows, cols, ldw, counts, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "se12_encode_histogram");
  return SE12_OK;
}

int se12_codebook_from_counts(const uint32_t* counts, uint8_t* codebook) {
  if (!counts || !codebook) return fail(SE12_ERR_INVALID_ARGUMENT, "null argument");
  int order[256];
  for (int i = 0; i < 256; ++i) order[i] = i;
  std::sort(order, order + 256, [&](int a, int b) {
    if (counts[a] != counts[b]) return counts[a] > counts[b];
    return a > b;  // equal counts: larger exponent first (stable argsort, reversed)
  });
  for (int i = 0; i < SE12_CODEBOOK_SIZE; ++i) codebook[i] = static_cast<uint8_t>(order[i]);
  return SE12_OK;
}

int se12_encode_tiles(const uint16_t* w, int rows, int cols, int ldw, const uint8_t* codebook, uint8_t* sm,
                      uint8_t* ec, uint8_t* esc, uint8_t* tile_fallback, void* stream) {
  if (!w || !codebook || !sm || !ec || !esc || !tile_fallback || rows <= 0 || cols <= 0 || ldw < cols)
    return fail(SE12_ERR_INVALID_ARGUMENT, "bad arguments");
  if (!aligned16(sm) || !aligned16(ec)) return fail(SE12_ERR_MISALIGNED, "sm and ec must be 16-byte aligned");
  cudaError_t err = se12::launch_encode_tiles(w, rows, cols, ldw, codebook, sm, ec, esc, tile_fallback,
                                              static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "se12_encode_tiles");
  return SE12_OK;
}

int se12_encode_bitmap(const uint8_t* tile_fallback, int tiles, uint8_t* bitmap, int32_t* fallback_index,
                       int32_t* fallback_count, void* stream) {
  if (!tile_fallback || !bitmap || !fallback_index || !fallback_count || tiles < 0)
    return fail(SE12_ERR_INVALID_ARGUMENT, "bad arguments");
  cudaError_t err = se12::launch_encode_bitmap(tile_fallback, tiles, bitmap, fallback_index, fallback_count,
                                               static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "se12_encode_bitmap");
  return SE12_OK;
}

int se12_encode_raw(const uint16_t* w, int rows, int cols, int ldw, const int32_t* fallback_index, int16_t* raw,
                    void* stream) {
  if (!w || !fallback_index || rows <= 0 || cols <= 0 || ldw < cols)
    return fail(SE12_ERR_INVALID_ARGUMENT, "bad arguments");
  cudaError_t err = se12::launch_encode_raw(w, rows, cols, ldw, fallback_index, reinterpret_cast<uint16_t*>(raw),
                                            static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "se12_encode_raw");
  return SE12_OK;
}

int se12_device_status(unsigned* status, int clear) {
  if (!status) return fail(SE12_ERR_INVALID_ARGUMENT, "null argument");
  cudaError_t err = se12::read_device_status(status, clear != 0);
  if (err != cudaSuccess) return cuda_fail(err, "read device status");
  return SE12_OK;
}

int se12_set_wait_limit_ns(unsigned long long ns) {
  if (ns < SE12_MIN_WAIT_LIMIT_NS || ns > SE12_MAX_WAIT_LIMIT_NS)
    return fail(SE12_ERR_INVALID_ARGUMENT, "wait limit must be in " + std::to_string(SE12_MIN_WAIT_LIMIT_NS) + ".." +
                                               std::to_string(SE12_MAX_WAIT_LIMIT_NS) + " ns");
  cudaError_t err = se12::set_wait_limit(ns);
  if (err != cudaSuccess) return cuda_fail(err, "set wait limit");
  return SE12_OK;
}

int se12_wait_limit_ns(unsigned long long* ns) {
  if (!ns) return fail(SE12_ERR_INVALID_ARGUMENT, "null argument");
  cudaError_t err = se12::get_wait_limit(ns);
  if (err != cudaSuccess) return cuda_fail(err, "read wait limit");
  return SE12_OK;
}

}  // extern "C"

// ------------------------------------------------------------------ chains
// A chain: GEMVs run in order by one persistent launch (se12_chain.cu).
// Host side: the ops (with their TMA descriptors) in a vector; upload copies
// them to a caller buffer on the device and zeroes the caller's workspace.
struct se12_chain {
  std::vector<se12::ChainOp> ops;
  std::vector<int> starts;  // [ops][sm_count + 1] CTA tile ranges (made at upload)
  int batch = 1;
  bool dense = false;
  int device = 0;
  int sm_count = 0;
  int consumers = 0;
  int x_bytes = 0;
  int x_stride_max = 0;
  int n_ar = 0;
  se12::PeerArgs peers{};
  void* desc_dev = nullptr;
  void* ws_dev = nullptr;
  bool uploaded = false;
};

namespace {

constexpr size_t kChainSmemLimit = 227 * 1024;
constexpr int kChainMinConsumers = 12;

// x budget: what is left of shared memory with kChainMinConsumers warps.
size_t chain_x_budget(bool dense, int batch) {
  return kChainSmemLimit - se12::chain_smem_bytes(dense, kChainMinConsumers, 0, batch);
}

// Consumer warps that fit beside an x buffer of x_bytes.
int chain_consumers(bool dense, int x_bytes, int batch) {
  int c = se12::kChainMaxWarps;
  while (c > 1 && se12::chain_smem_bytes(dense, c, x_bytes, batch) > kChainSmemLimit) --c;
  return c;
}

int chain_x_stride(int width_tiles) { return width_tiles * 512 + 64; }

// Tile columns per op so that batch rows of x fit the budget.
int chain_split_width(bool dense, int batch, int tile_cols) {
  const size_t budget = chain_x_budget(dense, batch);
  int w = tile_cols;
  while (w > 1 && static_cast<size_t>(batch) * chain_x_stride(w) > budget) w = (w + 1) / 2;
  return w;
}

struct ChainLayout {
  size_t done, gen, rowcnt, partials, total;
};

// Workspace: done[n_ops] | gen[2] | rowcnt[n_ops][grid][2] | partials[grid][2][256]
ChainLayout chain_layout(int n_ops, int grid) {
  ChainLayout l{};
  auto up = [](size_t v) { return (v + 255) / 256 * 256; };
  l.done = 0;
  l.gen = up(static_cast<size_t>(n_ops) * 4);
  l.rowcnt = l.gen + 256;
  l.partials = up(l.rowcnt + static_cast<size_t>(n_ops) * grid * 2 * 4);
  l.total = up(l.partials + static_cast<size_t>(grid) * 2 * 256 * 4);
  return l;
}

// The tile range of every CTA for one op (grid + 1 boundaries): whole tile
// rows per CTA when that costs no more than an even split of the tiles (the
// longest warp part in tiles, plus 2 for the cross-CTA sum a row split
// needs). Rows then never cross CTAs and are summed in shared memory.
void chain_starts(const se12::ChainOp& op, int grid, int consumers, int* st) {
  const long long W = op.k1 - op.k0, T = op.tiles, R = T / W, G = grid, C = consumers;
  const long long cost_rows = (((R + G - 1) / G) * W + C - 1) / C;
  const long long cost_split = ((T + G - 1) / G + C - 1) / C + 2;
  const bool by_rows = cost_rows <= cost_split;
  for (long long c = 0; c <= G; ++c) st[c] = static_cast<int>(by_rows ? (R * c / G) * W : T * c / G);
}

int chain_check_open(se12_chain* c) {
  if (!c) return fail(SE12_ERR_INVALID_ARGUMENT, "null chain");
  if (c->uploaded) return fail(SE12_ERR_INVALID_ARGUMENT, "the chain was uploaded: no more ops can be added");
  if (static_cast<int>(c->ops.size()) >= se12::kChainMaxOps)
    return fail(SE12_ERR_INVALID_ARGUMENT, "a chain holds at most " + std::to_string(se12::kChainMaxOps) + " ops");
  return SE12_OK;
}

// Appends the op(s) of one GEMV: one per column block of x that fits the
// shared-memory budget; every block after the first accumulates into y.
int chain_append(se12_chain* c, se12::ChainOp base, int tile_cols, int cols) {
  const int width = chain_split_width(c->dense, c->batch, tile_cols);
  const int tile_rows_n = base.tiles;  // caller passes tile rows here
  for (int k0 = 0; k0 < tile_cols; k0 += width) {
    se12::ChainOp op = base;
    op.k0 = k0;
    op.k1 = std::min(tile_cols, k0 + width);
    op.tiles = tile_rows_n * (op.k1 - op.k0);
    op.x_cols = std::min(cols, op.k1 * SE12_TILE_COLS) - k0 * SE12_TILE_COLS;
    op.accumulate = k0 > 0 ? 1 : 0;
    c->x_stride_max = std::max(c->x_stride_max, chain_x_stride(op.k1 - op.k0));
    c->ops.push_back(op);
  }
  return SE12_OK;
}

int chain_check_io(se12_chain* c, int rows, int cols, const uint16_t* x, int ldx, const float* y, int ldy) {
  return check_gemv_io(rows, cols, x, c->batch, ldx, y, ldy);
}

}  // namespace

extern "C" {

size_t se12_tile_records_bytes(int rows, int cols) {
  if (rows <= 0 || cols <= 0) return 0;
  return static_cast<size_t>(tiles_of(rows, cols)) * SE12_ESCAPE_BUDGET * sizeof(uint32_t);
}

int se12_matrix_prepare_records(const se12_matrix* m, uint32_t* records, void* stream) {
  if (!m || !records) return fail(SE12_ERR_INVALID_ARGUMENT, "null argument");
  if (!aligned16(records)) return fail(SE12_ERR_MISALIGNED, "records must be 16-byte aligned");
  cudaError_t err = se12::launch_prepare_records(m->view, records, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "se12_matrix_prepare_records launch");
  return SE12_OK;
}

int se12_chain_create(int batch, int dense, se12_chain** out) {
  if (!out) return fail(SE12_ERR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  if (batch < 1 || batch > SE12_MAX_BATCH)
    return fail(SE12_ERR_INVALID_ARGUMENT, "batch must be in 1.." + std::to_string(SE12_MAX_BATCH));
  int device = 0, sm_count = 0;
  int st = current_device_info(&device, &sm_count);
  if (st != SE12_OK) return st;
  se12_chain* c = new se12_chain();
  c->batch = batch;
  c->dense = dense != 0;
  c->device = device;
  c->sm_count = sm_count;
  c->peers.world = 1;
  *out = c;
  return SE12_OK;
}

void se12_chain_destroy(se12_chain* c) { delete c; }

static int chain_add_se12(se12_chain* c, const se12_matrix* m, const uint32_t* records, const uint16_t* x, int ldx,
                          float* y, int ldy, int ar_index) {
  int st = chain_check_open(c);
  if (st != SE12_OK) return st;
  if (c->dense) return fail(SE12_ERR_INVALID_ARGUMENT, "a dense chain takes dense GEMVs only");
  if (!m || !records) return fail(SE12_ERR_INVALID_ARGUMENT, "null matrix or records");
  if (m->device != c->device) return fail(SE12_ERR_INVALID_ARGUMENT, "matrix and chain are on different devices");
  if (!aligned16(records)) return fail(SE12_ERR_MISALIGNED, "records must be 16-byte aligned");
  st = chain_check_io(c, m->view.rows, m->view.cols, x, ldx, y, ldy);
  if (st != SE12_OK) return st;
  const se12::MatrixView& v = m->view;
  se12::ChainOp op{};
  // one-tile boxes of the sm and ec streams
  const cuuint64_t rows16 = static_cast<cuuint64_t>(v.tiles) * SE12_TILE_ROWS;
  const cuuint64_t sm_dims[3] = {128, 2, rows16};
  const cuuint64_t sm_strides[2] = {128, 256};
  const cuuint32_t sm_box[3] = {128, 2, SE12_TILE_ROWS};
  st = encode_map(&op.sm_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, v.sm, sm_dims, sm_strides, sm_box);
  if (st != SE12_OK) return st;
  const cuuint64_t ec_dims[2] = {128, rows16};
  const cuuint64_t ec_strides[1] = {128};
  const cuuint32_t ec_box[2] = {128, SE12_TILE_ROWS};
  st = encode_map(&op.ec_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, v.ec, ec_dims, ec_strides, ec_box);
  if (st != SE12_OK) return st;
  op.records = records;
  op.fallback_raw = v.fallback_raw;
  op.x = x;
  op.y = y;
  op.ldx = ldx;
  op.ldy = ldy;
  op.rows = v.rows;
  op.cols = v.cols;
  op.tile_cols = v.tile_cols;
  op.tiles = v.tile_rows;  // tile rows: chain_append multiplies by the block width
  op.ar_index = ar_index;
  op.segments = v.segments;
  for (int s = 0; s < se12::kMaxSegments; ++s) {
    op.seg_end[s] = v.seg_end[s];
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    for (int code = 0; code < 16; ++code) w[code >> 2] |= se12::table_byte(v.codebooks[s], code) << (8 * (code & 3));
    for (int q = 0; q < 4; ++q) op.tab[s][q] = w[q];
  }
  return chain_append(c, op, v.tile_cols, v.cols);
}

int se12_chain_add_gemv(se12_chain* c, const se12_matrix* m, const uint32_t* records, const uint16_t* x, int ldx,
                        float* y, int ldy) {
  return chain_add_se12(c, m, records, x, ldx, y, ldy, -1);
}

int se12_chain_add_gemv_allreduce(se12_chain* c, const se12_matrix* m, const uint32_t* records, const uint16_t* x,
                                  int ldx, float* y, int ldy, const se12_peer_group* g) {
  int st = chain_check_open(c);
  if (st != SE12_OK) return st;
  if (!g) return fail(SE12_ERR_INVALID_ARGUMENT, "null peer group");
  if (g->world < 2 || g->world > SE12_MAX_PEERS || g->rank < 0 || g->rank >= g->world)
    return fail(SE12_ERR_INVALID_ARGUMENT, "peer group needs 2.." + std::to_string(SE12_MAX_PEERS) +
                                               " ranks and 0 <= rank < world");
  if (!m) return fail(SE12_ERR_INVALID_ARGUMENT, "null matrix");
  if (m->view.rows > g->rows_cap)
    return fail(SE12_ERR_INVALID_ARGUMENT, "matrix has " + std::to_string(m->view.rows) +
                                               " rows, the peer buffers hold " + std::to_string(g->rows_cap));
  if (chain_split_width(false, c->batch, m->view.tile_cols) < m->view.tile_cols)
    return fail(SE12_ERR_INVALID_ARGUMENT, "an all-reduced GEMV must fit one op: x of this batch and width is "
                                           "too large for shared memory");
  for (int r = 0; r < g->world; ++r)
    if (!g->recv[r] || !aligned16(g->recv[r])) return fail(SE12_ERR_MISALIGNED, "null or misaligned peer buffer");
  if (c->n_ar > 0) {
    if (c->peers.world != g->world || c->peers.rank != g->rank || c->peers.rows_cap != g->rows_cap)
      return fail(SE12_ERR_INVALID_ARGUMENT, "all all-reduced ops of a chain use one peer group");
    for (int r = 0; r < g->world; ++r)
      if (c->peers.recv[r] != static_cast<unsigned long long*>(g->recv[r]))
        return fail(SE12_ERR_INVALID_ARGUMENT, "all all-reduced ops of a chain use one peer group");
  } else {
    c->peers.world = g->world;
    c->peers.rank = g->rank;
    c->peers.rows_cap = g->rows_cap;
    for (int r = 0; r < g->world; ++r) c->peers.recv[r] = static_cast<unsigned long long*>(g->recv[r]);
    c->peers.epoch = g->epoch;
  }
  st = chain_add_se12(c, m, records, x, ldx, y, ldy, c->n_ar);
  if (st == SE12_OK) ++c->n_ar;
  return st;
}

int se12_chain_add_dense(se12_chain* c, const uint16_t* w, int rows, int cols, int ldw, const uint16_t* x, int ldx,
                         float* y, int ldy) {
  int st = chain_check_open(c);
  if (st != SE12_OK) return st;
  if (!c->dense) return fail(SE12_ERR_INVALID_ARGUMENT, "an SE12 chain takes SE12 GEMVs only");
  if (!w) return fail(SE12_ERR_INVALID_ARGUMENT, "null weights");
  if (rows <= 0 || cols <= 0 || ldw < cols) return fail(SE12_ERR_INVALID_ARGUMENT, "bad weight shape");
  if (!aligned16(w) || (ldw % 8) != 0) return fail(SE12_ERR_MISALIGNED, "W must be 16-byte aligned, ldw % 8 == 0");
  st = chain_check_io(c, rows, cols, x, ldx, y, ldy);
  if (st != SE12_OK) return st;
  se12::ChainOp op{};
  int raw_3d = 0;
  st = encode_raw_map(&op.sm_map, w, rows, cols, ldw, &raw_3d);
  if (st != SE12_OK) return st;
  op.raw_3d = raw_3d;
  op.x = x;
  op.y = y;
  op.ldx = ldx;
  op.ldy = ldy;
  op.rows = rows;
  op.cols = cols;
  op.tile_cols = (cols + SE12_TILE_COLS - 1) / SE12_TILE_COLS;
  op.tiles = (rows + SE12_TILE_ROWS - 1) / SE12_TILE_ROWS;
  op.ar_index = -1;
  op.segments = 1;
  for (int s = 0; s < se12::kMaxSegments; ++s) op.seg_end[s] = INT32_MAX;
  return chain_append(c, op, op.tile_cols, cols);
}

int se12_chain_ops(const se12_chain* c) { return c ? static_cast<int>(c->ops.size()) : 0; }

// Descriptors: the ops, then every op's CTA boundaries (int32 [n_ops][grid + 1]).
size_t se12_chain_descriptor_bytes(const se12_chain* c) {
  return c ? c->ops.size() * (sizeof(se12::ChainOp) + static_cast<size_t>(c->sm_count + 1) * sizeof(int)) : 0;
}

static void chain_finalize(se12_chain* c) {
  c->x_bytes = c->batch * c->x_stride_max;
  c->consumers = chain_consumers(c->dense, c->x_bytes, c->batch);
}

size_t se12_chain_workspace_bytes(const se12_chain* c) {
  if (!c || c->ops.empty()) return 0;
  se12_chain tmp = *c;
  chain_finalize(&tmp);
  return chain_layout(static_cast<int>(c->ops.size()), c->sm_count).total;
}

int se12_chain_upload(se12_chain* c, void* descriptors, void* workspace, size_t workspace_bytes, void* stream) {
  if (!c) return fail(SE12_ERR_INVALID_ARGUMENT, "null chain");
  if (c->ops.empty()) return fail(SE12_ERR_INVALID_ARGUMENT, "empty chain");
  if (!descriptors || (reinterpret_cast<uintptr_t>(descriptors) & 63u))
    return fail(SE12_ERR_MISALIGNED, "the descriptor buffer must be 64-byte aligned");
  chain_finalize(c);
  const ChainLayout l = chain_layout(static_cast<int>(c->ops.size()), c->sm_count);
  if (!workspace || workspace_bytes < l.total || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(SE12_ERR_WORKSPACE_TOO_SMALL, "chain workspace needs " + std::to_string(l.total) +
                                                  " bytes, 256-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t ops_bytes = c->ops.size() * sizeof(se12::ChainOp);
  c->starts.assign(c->ops.size() * static_cast<size_t>(c->sm_count + 1), 0);
  for (size_t j = 0; j < c->ops.size(); ++j)
    chain_starts(c->ops[j], c->sm_count, c->consumers, c->starts.data() + j * static_cast<size_t>(c->sm_count + 1));
  cudaError_t err = cudaMemcpyAsync(descriptors, c->ops.data(), ops_bytes, cudaMemcpyHostToDevice, s);
  if (err != cudaSuccess) return cuda_fail(err, "chain descriptor copy");
  err = cudaMemcpyAsync(static_cast<char*>(descriptors) + ops_bytes, c->starts.data(), c->starts.size() * sizeof(int),
                        cudaMemcpyHostToDevice, s);
  if (err != cudaSuccess) return cuda_fail(err, "chain descriptor copy");
  err = cudaMemsetAsync(workspace, 0, l.total, s);
  if (err != cudaSuccess) return cuda_fail(err, "chain workspace clear");
  c->desc_dev = descriptors;
  c->ws_dev = workspace;
  c->uploaded = true;
  return SE12_OK;
}

int se12_chain_reset(const se12_chain* c, void* stream) {
  if (!c || !c->uploaded) return fail(SE12_ERR_INVALID_ARGUMENT, "chain not uploaded");
  const ChainLayout l = chain_layout(static_cast<int>(c->ops.size()), c->sm_count);
  cudaError_t err = cudaMemsetAsync(c->ws_dev, 0, l.total, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "chain workspace clear");
  return SE12_OK;
}

int se12_chain_info(const se12_chain* c, int* grid, int* consumers, int* smem_bytes, int* ops) {
  if (!c || !grid || !consumers || !smem_bytes || !ops) return fail(SE12_ERR_INVALID_ARGUMENT, "null argument");
  se12_chain tmp = *c;
  chain_finalize(&tmp);
  *grid = tmp.sm_count;
  *consumers = tmp.consumers;
  *smem_bytes = static_cast<int>(se12::chain_smem_bytes(tmp.dense, tmp.consumers, tmp.x_bytes, tmp.batch));
  *ops = static_cast<int>(tmp.ops.size());
  return SE12_OK;
}

int se12_chain_run(const se12_chain* c, void* stream) {
  if (!c || !c->uploaded) return fail(SE12_ERR_INVALID_ARGUMENT, "chain not uploaded");
  int device = -1;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetDevice");
  if (device != c->device) return fail(SE12_ERR_INVALID_ARGUMENT, "the current device is not the chain's device");
  const int n = static_cast<int>(c->ops.size());
  const ChainLayout l = chain_layout(n, c->sm_count);
  char* ws = static_cast<char*>(c->ws_dev);
  se12::ChainParams p{};
  p.ops = static_cast<const se12::ChainOp*>(c->desc_dev);
  p.starts = reinterpret_cast<const int*>(static_cast<const char*>(c->desc_dev) + c->ops.size() * sizeof(se12::ChainOp));
  p.n_ops = n;
  p.batch = c->batch;
  p.consumers = c->consumers;
  p.x_stride = c->x_stride_max;
  p.x_bytes = c->x_bytes;
  p.n_ar = c->n_ar;
  p.done = reinterpret_cast<unsigned*>(ws + l.done);
  p.gen = reinterpret_cast<unsigned*>(ws + l.gen);
  p.rowcnt = reinterpret_cast<unsigned*>(ws + l.rowcnt);
  p.partials = reinterpret_cast<float*>(ws + l.partials);
  p.peers = c->peers;
  const size_t smem = se12::chain_smem_bytes(c->dense, c->consumers, c->x_bytes, c->batch);
  err = se12::launch_chain(c->dense, p, c->sm_count, smem, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "se12_chain_run launch");
  return SE12_OK;
}

}  // extern "C"
