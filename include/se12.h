/*
 * se12.h -- C ABI of the B200-native SE12 decode + GEMV library
 * (libse12_b200.so, built for sm_100a).
 *
 * SE12 stores every BF16 weight losslessly in about 12 bits: one
 * sign|mantissa byte plus a 4-bit code into a 15-entry exponent codebook,
 * per 16x256 tile up to 16 escaped exponents, and raw storage for tiles with
 * more escapes. These entry points replace the reference implementation's
 * GPU path (Acaua-Rangel/se12, package `lws`); each declaration cites the
 * reference interface it replaces as file:line within that project.
 *
 * Conventions
 *  - All pointers named *_dev or documented "device" are CUDA device
 *    pointers; `stream` is a cudaStream_t passed as void* (NULL = default).
 *  - Functions return an se12_status (0 = SE12_OK). On failure
 *    se12_last_error() returns a message for the calling thread.
 *  - No entry point allocates device memory or synchronises the stream:
 *    every buffer (outputs, workspaces, derived tables) is caller-owned.
 *    Launches are asynchronous on `stream`.
 *  - BF16 values travel as their uint16 bit patterns.
 */
#ifndef SE12_B200_H
#define SE12_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SE12_TILE_ROWS 16
#define SE12_TILE_COLS 256
#define SE12_ESCAPE_BUDGET 16
#define SE12_CODEBOOK_SIZE 15
#define SE12_FORMAT_VERSION 1
#define SE12_MAX_BATCH 16
#define SE12_MAX_SEGMENTS 4
#define SE12_MAX_PEERS 8

typedef enum se12_status {
  SE12_OK = 0,
  SE12_ERR_INVALID_ARGUMENT = 1,
  SE12_ERR_UNSUPPORTED_FORMAT = 2, /* tile shape, escape budget or format version (container.py:21-27) */
  SE12_ERR_MISALIGNED = 3,         /* a pointer / leading dimension breaks the alignment rule */
  SE12_ERR_WORKSPACE_TOO_SMALL = 4,
  SE12_ERR_CUDA = 5,               /* a CUDA runtime/driver call failed */
  SE12_ERR_UNSUPPORTED_DEVICE = 6, /* not a compute capability 10.0 (B200) device */
  SE12_ERR_DEVICE_FAULT = 7        /* a kernel recorded an error in the device status word */
} se12_status;

/*
 * The five SE12 streams of one matrix, already in device memory, exactly as
 * lws.pack writes them (src/lws/adapters/safetensors/packed_store.py:70-107):
 *   sm [T*4096] u8, ec [T*2048] u8, esc [T*16] u8,
 *   fallback_bitmap [ceil(T/8)] u8, fallback_raw [F*4096] i16,
 * with T = ceil(rows/16) * ceil(cols/256) tiles and F fallback tiles.
 * escape_pos and fallback_index are derived tables (sizes from
 * se12_escape_pos_bytes / se12_fallback_index_bytes) that
 * se12_matrix_prepare fills.
 * All stream and derived-table pointers must be 16-byte aligned.
 */
typedef struct se12_streams {
  int32_t rows, cols;
  int32_t tile_rows, tile_cols; /* format metadata: must be 16 and 256 */
  int32_t escape_budget;        /* must be 16 */
  int32_t format_version;       /* must be 1 */
  uint8_t codebook[SE12_CODEBOOK_SIZE];
  const uint8_t* sm;
  const uint8_t* ec;
  const uint8_t* esc;
  const uint8_t* fallback_bitmap;
  const int16_t* fallback_raw;
  uint16_t* escape_pos;   /* derived, caller-allocated: [T*16] */
  int32_t* fallback_index; /* derived, caller-allocated: [T rounded up to a multiple of 4] */
} se12_streams;

/* Opaque host-side handle: device pointers plus TMA descriptors. Immutable
 * after creation, so concurrent calls on different streams are safe. */
typedef struct se12_matrix se12_matrix;

/* Bytes of the two derived tables for a rows x cols matrix. */
size_t se12_escape_pos_bytes(int rows, int cols);
size_t se12_fallback_index_bytes(int rows, int cols);

/* Validates the streams' format and builds the handle (host only, no GPU work).
 * Replaces the upload / host precompute of Se12MatVecKernel.__init__ and
 * _upload_se12_streams (src/lws/adapters/cuda/gemv.py:183-194, 229-264). */
int se12_matrix_create(const se12_streams* streams, se12_matrix** out);

/* A segmented matrix: `streams` hold the tile-major concatenation of
 * `segments` (1..SE12_MAX_SEGMENTS) SE12 matrices with the same cols -- for
 * example the q, k and v projections of an attention block, or gate and up
 * of an MLP, which multiply the same x -- so that one se12_gemv computes all
 * of them into one y of sum(segment_rows) rows. Each segment keeps its own
 * codebook (codebooks: [segments][15]). streams->rows must equal
 * sum(segment_rows) and every segment but the last needs a multiple of 16
 * rows, so that the segments' tiles follow each other:
 *   sm, ec, esc, fallback_raw: the segments' streams one after the other;
 *   fallback_bitmap: the segments' tile bits one after the other, MSB first.
 * streams->codebook is ignored. Every entry point accepts the result like a
 * plain matrix. No reference counterpart (the reference launches one GEMV
 * per tensor). */
int se12_matrix_create_segmented(const se12_streams* streams, int segments, const int32_t* segment_rows,
                                 const uint8_t* codebooks, se12_matrix** out);

/* Fills escape_pos and fallback_index on the device (once per matrix).
 * Replaces the host prefix sums fallback_offsets / row_escape_offset
 * (src/lws/adapters/cuda/gemv.py:47-77). */
int se12_matrix_prepare(const se12_matrix* m, void* stream);

void se12_matrix_destroy(se12_matrix* m);

/* Workspace of se12_gemv for this matrix (any batch size). The workspace
 * must be zeroed once (se12_workspace_clear) before first use; every
 * completed call leaves it ready for the next. Its layout does not depend on
 * the matrix, so one workspace (sized for the largest matrix) serves every
 * call on a stream; calls that may overlap on the GPU need separate ones.
 * After se12_device_status reports a timed-out wait (bit 0), zero every
 * workspace that such a call used again before reusing it: a CTA that
 * published its partial row after its finisher gave up leaves its flag set. */
size_t se12_gemv_workspace_bytes(const se12_matrix* m, int batch);
int se12_workspace_clear(void* workspace_dev, size_t bytes, void* stream);

/* The launch se12_gemv makes for this matrix and batch: the fixed launch
 * table that replaces the reference's launch heuristic and tuner
 * (default_launch_configuration, src/lws/domain/launch/heuristic.py:46-51;
 * src/lws/tune.py:34-57). Informational: se12_gemv computes the same
 * configuration itself. */
typedef struct se12_launch_config {
  int grid;          /* CTAs */
  int threads;       /* per CTA */
  int smem_bytes;    /* dynamic shared memory per CTA */
  int ctas_per_sm;   /* CTAs the shared memory lets share an SM */
  int stage_tiles;   /* 16x256 tiles per pipeline stage (4 or 8) */
  int stages;        /* pipeline depth */
  int x_resident;    /* 1: all of x in shared memory; 0: staged per stage */
  int row_mode;      /* 1: whole tile rows per CTA; 0: stream-K with split rows */
  int wide;          /* 1: one CTA per SM whose warp groups take 4-tile stages in turn */
} se12_launch_config;

int se12_gemv_launch_config(const se12_matrix* m, int batch, se12_launch_config* out);

/* The same answer from the shape alone, for a device of sm_count SMs
 * (host only: no GPU, no matrix; what se12_gemv_launch_config returns for
 * a matrix of rows x cols on such a device). */
int se12_gemv_plan(int rows, int cols, int batch, int sm_count, se12_launch_config* out);

/*
 * Fused decode + GEMV:  y[b, n] = sum_k W[n, k] * x[b, k],  fp32 accumulate,
 * fp32 output. x: device BF16 [batch, ldx], y: device fp32 [batch, ldy].
 * 1 <= batch <= SE12_MAX_BATCH; x 16-byte aligned, ldx % 8 == 0 and
 * ldx >= cols rounded up to 8 (x[b, cols..ldx) may hold anything); ldy >= rows.
 * Replaces Se12MatVecKernel.multiply (src/lws/adapters/cuda/gemv.py:196-226)
 * and the kernel lws_gemv_se12 (src/lws/adapters/cuda/kernels/gemv_se12.cu:50-64).
 */
int se12_gemv(const se12_matrix* m, const uint16_t* x_dev, int batch, int ldx, float* y_dev, int ldy,
              void* workspace_dev, size_t workspace_bytes, void* stream);

/*
 * Fused GEMV + all-reduce for tensor parallelism with the input columns
 * sharded (the attention-output and MLP-down projections of a Megatron
 * split): every rank of a peer group calls it, in the same order, on its
 * column shard of the same rows x cols matrix, and each gets
 *   y = sum over ranks of (its shard's GEMV),
 * summed in rank order, so all ranks hold the same bits. No counterpart in
 * the reference, which runs on one GPU at a time
 * (.spec/features/fused-decode-gemv/spec.md:159); it replaces a GEMV
 * followed by an NCCL all-reduce: inside the GEMV kernel, each finished tile
 * row is stored into every rank's receive buffer over peer memory (NVLink),
 * every value in one 64-bit word with the call's epoch, and read back once
 * all ranks' words carry it.
 *
 * The group describes buffers every rank allocated and mapped into every
 * other rank (se12_ipc_handle / se12_ipc_open, or any peer mapping),
 * indexed by rank:
 *   recv[r]:  se12_peer_recv_bytes(world, rows_cap) bytes, 16-byte aligned,
 *             zeroed once;
 *   epoch:    this rank's own two int32 (call counter, CTAs finished),
 *             zeroed once, not shared with the other ranks.
 * All ranks must make the same sequence of calls on a group (the last CTA
 * of each call bumps the counter); a call waits (bounded, then reports
 * SE12_ERR_DEVICE_FAULT through se12_device_status) for every rank's rows.
 * Calls on one group must be ordered on one stream per rank.
 */
typedef struct se12_peer_group {
  int32_t world, rank, rows_cap;
  void* recv[SE12_MAX_PEERS];
  int32_t* epoch;
} se12_peer_group;

/* Mapping another process's device buffer (CUDA IPC), for the peer group's
 * buffers: se12_ipc_handle gives the 64-byte handle of the allocation that
 * holds dev_ptr and dev_ptr's offset in it; se12_ipc_open maps it on the
 * current device (enabling peer access) and returns the pointer for that
 * offset plus the mapping to pass to se12_ipc_close. An allocation can be
 * opened once per process. */
int se12_ipc_handle(const void* dev_ptr, uint8_t* handle_out /* [64] */, uint64_t* offset_out);
int se12_ipc_open(const uint8_t* handle /* [64] */, uint64_t offset, void** dev_ptr_out, void** mapping_out);
int se12_ipc_close(void* mapping);

size_t se12_peer_recv_bytes(int world, int rows_cap);
int se12_gemv_allreduce(const se12_matrix* m, const uint16_t* x_dev, int batch, int ldx, float* y_dev, int ldy,
                        void* workspace_dev, size_t workspace_bytes, const se12_peer_group* peers, void* stream);

/*
 * Fused GEMV + all-gather for tensor parallelism with the output rows
 * sharded (every GEMV row-sharded, the whole output wanted on every rank):
 * this rank's matrix holds rows row0 .. row0 + rows - 1 of a rows_full-row
 * output, and every rank gets the whole output in y_dev [batch][ldy >=
 * rows_full]. No counterpart in the reference (one GPU at a time); it
 * replaces a GEMV followed by an NCCL all-gather: each finished tile row
 * is stored into every rank's receive buffer at its place in the whole
 * output (each value with the call's epoch in one 64-bit word), and every
 * CTA then unpacks its slice of the whole output once the words carry the
 * epoch. Same peer group, ordering and error rules as se12_gemv_allreduce
 * (the two share the group's call counter); needs rows_full <= world x
 * rows_cap.
 */
int se12_gemv_allgather(const se12_matrix* m, const uint16_t* x_dev, int batch, int ldx, float* y_dev, int ldy, int row0,
                        int rows_full, void* workspace_dev, size_t workspace_bytes, const se12_peer_group* peers,
                        void* stream);

/*
 * se12_gemv without a caller workspace, for callers that cannot allocate
 * device memory: a host that has reserved all of HBM for its own arena (so
 * cudaMalloc fails), or a binding that holds no device buffer it could keep
 * alive and zeroed between calls. It has no counterpart in the reference.
 * Same arguments, result and errors as se12_gemv, except:
 *  - The scratch is a fixed 644 KiB array in the library's device image,
 *    held by every GPU that loads the library until the process exits: the
 *    partial rows and flags of up to 320 CTAs (two per SM on up to 160
 *    SMs). A launch that would need more returns SE12_ERR_UNSUPPORTED_DEVICE,
 *    and a batch above SE12_MAX_BATCH SE12_ERR_INVALID_ARGUMENT, each with a
 *    message and without launching anything. Matrix size is not limited.
 *  - The current device must be the matrix's device. The first call on a
 *    device looks up the scratch's address (cudaGetSymbolAddress); make that
 *    first call before any stream capture. The address is kept for the life
 *    of the process: after cudaDeviceReset (or anything else that replaces
 *    the device's primary context) this entry point must not be called
 *    again on that device in the same process.
 *  - Every call clears the scratch's flags on `stream` (cudaMemsetAsync)
 *    and then launches the GEMV; it allocates nothing.
 *  - All calls on a device share the one scratch, which keeps the last
 *    call's contents: calls that can overlap on the GPU (on different
 *    streams without ordering between them) race and give wrong results.
 */
int se12_gemv_noalloc(const se12_matrix* m, const uint16_t* x_dev, int batch, int ldx, float* y_dev, int ldy,
                      void* stream);

/*
 * Chains: a sequence of GEMVs run in order by ONE persistent launch, for
 * example every projection of a decode step (q/k/v, o, gate/up, down of each
 * layer, then the LM head). Op j reads its x only after op j - 1 has been
 * completed by every CTA (so x of op j may be y of op j - 1, or computed from
 * it between launches), while the weights of op j already stream in: the
 * per-launch fill, drain and hand-over cost of one launch per GEMV is paid
 * once per chain. Results are the same GEMVs as se12_gemv's (fp32
 * accumulation, fp32 y; within 1e-3 of the fp64 product), deterministic for
 * a given chain. This is the stacked mode of the reference's
 * microbenchmark design (.spec/features/fused-decode-gemv/design.md:155-165:
 * the same projections of every layer back to back), taken into one kernel;
 * each op replaces one Se12MatVecKernel.multiply / lws_gemv_se12 call
 * (src/lws/adapters/cuda/gemv.py:196-226, kernels/gemv_se12.cu:50-64).
 *
 * Use: se12_chain_create -> se12_chain_add_* per GEMV, in order ->
 * se12_chain_descriptor_bytes / se12_chain_workspace_bytes -> allocate both
 * (descriptors 64-byte aligned, workspace 256-byte aligned) ->
 * se12_chain_upload (copies the descriptors, zeroes the workspace) ->
 * se12_chain_run on a stream, any number of times (graph-capturable: it only
 * launches). Launches of one chain must be ordered on one stream. The chain
 * keeps the pointers it was given: matrices, records, x and y must stay
 * allocated while it runs. A chain's GEMVs all have the chain's batch; one
 * whose x (batch x cols BF16) does not fit shared memory is split by column
 * blocks into ops that accumulate into y. After se12_device_status reports a
 * timed-out wait, se12_chain_reset zeroes the workspace before the next run.
 */
typedef struct se12_chain se12_chain;

/* Per-tile records a chain reads (escape positions with their exponents,
 * fallback ranks): 64 bytes per tile, filled once per matrix by
 * se12_matrix_prepare_records after se12_matrix_prepare. No reference
 * counterpart (derived like the reference's host tables, gemv.py:47-77). */
size_t se12_tile_records_bytes(int rows, int cols);
int se12_matrix_prepare_records(const se12_matrix* m, uint32_t* records_dev, void* stream);

/* dense = 1: a chain of dense BF16 GEMVs (the comparison baseline, the
 * chain form of bf16_gemv / lws_gemv_raw_bf16, gemv_raw_bf16.cu:18-56). */
int se12_chain_create(int batch, int dense, se12_chain** out);
int se12_chain_add_gemv(se12_chain* c, const se12_matrix* m, const uint32_t* records_dev, const uint16_t* x_dev,
                        int ldx, float* y_dev, int ldy);
/* The GEMV of a column shard, its rows all-reduced over the peer group (as
 * se12_gemv_allreduce). Every rank's chain must hold the same ops in the same
 * order; all such ops of a chain use one peer group. */
int se12_chain_add_gemv_allreduce(se12_chain* c, const se12_matrix* m, const uint32_t* records_dev,
                                  const uint16_t* x_dev, int ldx, float* y_dev, int ldy, const se12_peer_group* peers);
int se12_chain_add_dense(se12_chain* c, const uint16_t* w_dev, int rows, int cols, int ldw, const uint16_t* x_dev,
                         int ldx, float* y_dev, int ldy);
int se12_chain_ops(const se12_chain* c);
size_t se12_chain_descriptor_bytes(const se12_chain* c);
size_t se12_chain_workspace_bytes(const se12_chain* c);
int se12_chain_upload(se12_chain* c, void* descriptors_dev, void* workspace_dev, size_t workspace_bytes, void* stream);
int se12_chain_run(const se12_chain* c, void* stream);
int se12_chain_reset(const se12_chain* c, void* stream);
/* The launch se12_chain_run makes: CTAs, consumer warps per CTA, dynamic
 * shared memory, ops (after column splits). */
int se12_chain_info(const se12_chain* c, int* grid, int* consumers, int* smem_bytes, int* ops);
void se12_chain_destroy(se12_chain* c);

/* Exact BF16 bits of the whole matrix, row-major [rows, ldo] (ldo >= cols).
 * Replaces CudaSe12WeightDecoder.decode / decode_to_device and the kernel
 * lws_se12_decode (src/lws/adapters/cuda/se12_decoder.py:54-76,
 * src/lws/adapters/cuda/kernels/se12_decode.cu:12-22). */
int se12_decode(const se12_matrix* m, uint16_t* out_dev, int ldo, void* stream);

/* Exact BF16 bits of the requested rows (device int32 [nrows], any order,
 * repeats allowed) into out[i, :] (row-major [nrows, ldo]). An out-of-range
 * row index sets SE12_ERR_DEVICE_FAULT in the device status.
 * Replaces CudaSe12WeightDecoder.decode_rows (src/lws/adapters/cuda/se12_decoder.py:64-70). */
int se12_decode_rows(const se12_matrix* m, const int32_t* rows_dev, int nrows, uint16_t* out_dev, int ldo,
                     void* stream);

/* Dense BF16 GEMV baseline over a row-major BF16 matrix W [rows, ldw] with
 * the same pipeline and output contract as se12_gemv (ldw % 8 == 0, W
 * 16-byte aligned). Replaces RawBf16MatVecKernel.multiply and lws_gemv_raw_bf16
 * (src/lws/adapters/cuda/gemv.py:143-172, src/lws/adapters/cuda/kernels/gemv_raw_bf16.cu:18-25). */
/* The launch bf16_gemv makes for a shape on a GPU with sm_count SMs (host
 * only), the dense counterpart of se12_gemv_plan. */
int bf16_gemv_plan(int rows, int cols, int batch, int sm_count, se12_launch_config* out);

/* se12_gemv launched with the configuration bf16_gemv picks for the same
 * shape (grid, stages, x placement, row mode or stream-K), so that both
 * kernels reduce in the same order: the order-matched configuration of the
 * reference's fused-GEMV spec (.spec/features/fused-decode-gemv/spec.md:89-94,
 * AC-032). On a matrix whose escaped weights all have exponent 0 (zeros and
 * subnormals) it returns the same bits as bf16_gemv on the decoded weights;
 * an escape with a non-zero exponent is added outside the tensor-core sum
 * and may round differently. Same arguments and workspace as se12_gemv. */
int se12_gemv_order_matched(const se12_matrix* m, const uint16_t* x_dev, int batch, int ldx, float* y_dev, int ldy,
                            void* workspace_dev, size_t workspace_bytes, void* stream);
size_t bf16_gemv_workspace_bytes(int rows, int cols, int batch);
int bf16_gemv(const uint16_t* w_dev, int rows, int cols, int ldw, const uint16_t* x_dev, int batch, int ldx,
              float* y_dev, int ldy, void* workspace_dev, size_t workspace_bytes, void* stream);

/*
 * Encoder (packer), byte-identical to the reference encode_tensor
 * (src/lws/domain/se12/codec.py:111-141). Input: device BF16 [rows, ldw].
 *  1. se12_encode_histogram: 256 exponent counts (device u32[256]).
 *  2. se12_codebook_from_counts: host, the 15 most frequent exponents,
 *     ties to the larger exponent (src/lws/domain/se12/codebook.py:41-59).
 *  3. se12_encode_tiles: sm, ec, esc and a per-tile fallback flag (u8[T]).
 *  4. se12_encode_bitmap: fallback bitmap, fallback_index [T] (-1 for
 *     non-fallback tiles) and the fallback tile count (device int32).
 *  5. se12_encode_raw: raw bits of the fallback tiles (fallback_raw [F*4096]).
 */
int se12_encode_histogram(const uint16_t* w_dev, int rows, int cols, int ldw, uint32_t* counts_dev, void* stream);
int se12_codebook_from_counts(const uint32_t* counts_host, uint8_t* codebook_out);
int se12_encode_tiles(const uint16_t* w_dev, int rows, int cols, int ldw, const uint8_t* codebook_host,
                      uint8_t* sm_dev, uint8_t* ec_dev, uint8_t* esc_dev, uint8_t* tile_fallback_dev, void* stream);
int se12_encode_bitmap(const uint8_t* tile_fallback_dev, int tiles, uint8_t* bitmap_dev, int32_t* fallback_index_dev,
                       int32_t* fallback_count_dev, void* stream);
int se12_encode_raw(const uint16_t* w_dev, int rows, int cols, int ldw, const int32_t* fallback_index_dev,
                    int16_t* raw_dev, void* stream);

/* Device status word (bit 0: a bounded wait timed out, bit 1: bad argument
 * seen by a kernel). Reading it synchronises with the device. While bit 0 is
 * set, the waits on other CTAs' and other GPUs' progress give up at once
 * instead of waiting out their limit (a lost peer ends the kernel after one
 * limit): clear it (clear = 1) and zero the workspaces the failed calls used
 * (se12_workspace_clear, se12_chain_reset) before the next calls. No
 * counterpart in the reference, whose kernels never wait on other blocks. */
int se12_device_status(unsigned* status_out, int clear);

/* Limit of those waits on the current device, in ns (default 2 s). A short
 * limit makes a wait on a peer that will not write run out quickly (for
 * failure-detection tests); a correct wait completes in microseconds. A
 * synchronous copy to the device. */
#define SE12_MIN_WAIT_LIMIT_NS 100000ull
#define SE12_MAX_WAIT_LIMIT_NS 60000000000ull
int se12_set_wait_limit_ns(unsigned long long ns);
int se12_wait_limit_ns(unsigned long long* ns_out);

const char* se12_status_string(int status);
const char* se12_last_error(void);
int se12_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* SE12_B200_H */
