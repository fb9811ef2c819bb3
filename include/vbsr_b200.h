/*
 * vbsr_b200.h — C ABI of the B200-native variable-block sparse-row (VBSR) SpMM engine.
 *
 * Computes FP32, non-transpose C = A * B where A is a packed VBSR matrix (block heights and
 * widths independently in {8,16,...,64}, blocks column-major, packed in row order) and B, C are
 * dense column-major panels of width 8, 16, 32 or 64 (leading dimensions K and M, the scalar
 * column and row counts of A).
 *
 * Every entry point takes plain pointers and sizes and returns a vbsr_status. On failure a
 * human-readable message is kept per host thread and returned by vbsr_get_last_error().
 *
 * Reference interface each entry point replaces (King-Clawthorne/VarBlockSpMM):
 *   vbsr_host_validate          HostMatrix::validate        include/varblockspmm/vbsr.hpp:28,
 *                                                           src/format/vbsr.cpp:29-82
 *   vbsr_matrix_create          Matrix::Matrix(HostMatrix)  vbsr.hpp:44, vbsr.cpp:84-113
 *   vbsr_matrix_destroy         Matrix::~Matrix / release   vbsr.hpp:45, vbsr.cpp:114-127
 *   vbsr_matrix_device_view     Matrix::device_view         vbsr.hpp:51, vbsr.cpp:163-166
 *   vbsr_matrix_info            Matrix::scalar_rows/cols    vbsr.hpp:52-53
 *   vbsr_plan_create            Plan::Plan                  vbsr.hpp:106, src/plan/plan.cpp:5-18
 *   vbsr_plan_execute           Plan::execute               vbsr.hpp:110, plan.cpp:19-22
 *   vbsr_plan_launch_count      Plan::launch_count          vbsr.hpp:112, plan.cpp:23-31
 *   vbsr_launch_row_owned       launch_row_owned            vbsr.hpp:158-159,
 *                                                           src/kernels/row_owned.cu:397-423
 *   vbsr_launch_row_owned_scalar launch_row_owned_scalar    vbsr.hpp:161, row_owned.cu:376-395
 *   vbsr_generate               generate(GeneratorOptions)  vbsr.hpp:69-80,
 *                                                           src/format/generator.cpp:7-88
 * Entry points with no single reference counterpart (the multi-GPU block-row partition and
 * multi-GPU plan, the on-device value generator, plan diagnostics) say so in their comments.
 */
#ifndef VBSR_B200_H
#define VBSR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VBSR_B200_ABI_VERSION 1

/* Status codes. The C++ drop-in header maps INVALID_ARGUMENT to std::invalid_argument and every
 * other non-OK code to std::runtime_error, as the reference does (vbsr.cpp:13-17,32-80;
 * plan.cpp:9-17; row_owned.cu:367-372). */
typedef enum vbsr_status {
  VBSR_OK = 0,
  VBSR_INVALID_ARGUMENT = 1, /* malformed matrix, bad RHS width, rejected kernel, bad sizes */
  VBSR_CUDA_ERROR = 2,       /* a CUDA runtime call failed; message is cudaGetErrorString  */
  VBSR_TIMEOUT = 3,          /* a bounded in-kernel wait gave up (pipeline stalled)         */
  VBSR_BOUNDS_VIOLATION = 4, /* the bounds-checked kernel found an out-of-range index      */
  VBSR_OUT_OF_MEMORY = 5     /* host allocation failed                                     */
} vbsr_status;

/* cudaStream_t is a pointer to this opaque driver type; callers may pass a cudaStream_t, a
 * torch.cuda.Stream.cuda_stream integer, or NULL for the legacy default stream. */
typedef struct CUstream_st* vbsr_stream_t;

/* Non-owning view of a host VBSR matrix: the fields of HostMatrix (vbsr.hpp:16-29) as pointers
 * plus element counts, so that the size checks of HostMatrix::validate can be restated. */
typedef struct vbsr_host_matrix_view {
  int32_t block_rows, block_cols;
  const int32_t* row_ptr;        size_t row_ptr_len;        /* block_rows + 1            */
  const int32_t* block_col;      size_t block_col_len;      /* nnzb                      */
  const int32_t* row_size;       size_t row_size_len;       /* block_rows                */
  const int32_t* col_size;       size_t col_size_len;       /* block_cols                */
  const int64_t* row_scalar_off; size_t row_scalar_off_len; /* block_rows + 1            */
  const int64_t* col_scalar_off; size_t col_scalar_off_len; /* block_cols + 1            */
  const int64_t* value_off;      size_t value_off_len;      /* nnzb + 1                  */
  const float* values;           size_t values_len;         /* value_off[nnzb]; values may be
                                                               NULL only where stated    */
} vbsr_host_matrix_view;

/* Non-owning device view in the reference's own layout (DeviceMatrix, vbsr.hpp:32-38). The
 * pointers are device pointers owned by the vbsr_matrix they came from. `values` is in the
 * engine's re-laid-out block format, not the reference's column-major block layout: each h x w
 * block keeps its offset and size but is stored as w/8 consecutive 8-column groups, each h rows
 * x 8 floats (32 bytes per row) with the two 16-byte halves of row r exchanged when bit 2 of r
 * is set. The launchers below accept views produced by this library only. */
typedef struct vbsr_device_matrix {
  int32_t block_rows, block_cols, nnzb;
  int64_t scalar_rows, scalar_cols;
  const int32_t *row_ptr, *block_col, *row_size, *col_size;
  const int64_t *row_scalar_off, *col_scalar_off, *value_off;
  const float* values;
} vbsr_device_matrix;

typedef struct vbsr_matrix_info {
  int32_t block_rows, block_cols;
  int64_t nnzb;
  int64_t scalar_rows, scalar_cols; /* M and K */
  int64_t value_count;
  int64_t device_bytes;             /* bytes of device memory owned by the matrix */
  int32_t device;                   /* CUDA ordinal the matrix lives on           */
  int32_t row_begin, row_end;       /* block-row range of the source view it holds */
} vbsr_matrix_info;

typedef struct vbsr_matrix vbsr_matrix; /* owning device copy (Matrix) */
typedef struct vbsr_plan vbsr_plan;     /* execution plan (Plan)       */

/* ---- Errors ------------------------------------------------------------------------------- */

/* Message of the last failing call on this host thread ("" if none). Valid until the next call
 * on this thread. */
const char* vbsr_get_last_error(void);

/* ---- Host format -------------------------------------------------------------------------- */

/* HostMatrix::validate (vbsr.cpp:29-82): the same checks in the same order, with the same
 * messages. Returns VBSR_INVALID_ARGUMENT on the first failing check. */
vbsr_status vbsr_host_validate(const vbsr_host_matrix_view* host);

/* ---- Owning device matrix ----------------------------------------------------------------- */

/* Matrix::Matrix (vbsr.cpp:84-113): validates `host`, then builds the device format on
 * `device` (-1 = the current device): the reference-layout metadata arrays, per-block and
 * per-row descriptors used by the kernels, and the values re-laid-out into 8-column groups by
 * an on-device kernel. Uploads are synchronous; the call returns when the matrix is usable from
 * any stream. */
vbsr_status vbsr_matrix_create(const vbsr_host_matrix_view* host, int device, vbsr_matrix** out);

/* Shard constructor for the multi-GPU block-row partition (no reference counterpart; the
 * reference is single-GPU): holds block rows [row_begin, row_end) of `host` as a matrix with
 * row_end - row_begin block rows and the full column structure. C for the shard has ld
 * M_r = row_scalar_off[row_end] - row_scalar_off[row_begin]; B is the full K x N panel. */
vbsr_status vbsr_matrix_create_rows(const vbsr_host_matrix_view* host, int32_t row_begin,
                                    int32_t row_end, int device, vbsr_matrix** out);

/* Like vbsr_matrix_create_rows, but `host->values` may be NULL: the values are produced on the
 * device by the engine's counter-based generator (vbsr_fill_uniform with stream
 * VBSR_STREAM_VALUES and `seed`), so a matrix of tens of GB needs no host copy. Value v of the
 * full matrix (packed index v) equals what vbsr_fill_uniform gives for index v. No reference
 * counterpart. */
vbsr_status vbsr_matrix_create_rows_generated(const vbsr_host_matrix_view* host, int32_t row_begin,
                                              int32_t row_end, uint64_t seed, int device,
                                              vbsr_matrix** out);

vbsr_status vbsr_matrix_destroy(vbsr_matrix* m);
vbsr_status vbsr_matrix_info_get(const vbsr_matrix* m, vbsr_matrix_info* out);
vbsr_status vbsr_matrix_device_view(const vbsr_matrix* m, vbsr_device_matrix* out);

/* ---- Plans -------------------------------------------------------------------------------- */

/* Kernel selection (Kernel, vbsr.hpp:91). SPLIT_ROW is rejected with VBSR_INVALID_ARGUMENT,
 * as plan.cpp:13-17 does. */
enum { VBSR_KERNEL_AUTO = 0, VBSR_KERNEL_ROW_OWNED = 1, VBSR_KERNEL_SPLIT_ROW = 2 };

/* Plan flags (no reference counterpart). */
enum {
  VBSR_PLAN_BOUNDS_CHECK = 1u << 0, /* use the bounds-checked kernel build                  */
  /* Keep every block row whole. By default a block row whose cost exceeds the fair share of one
   * SM (1/num_SMs of the matrix's) is cut into row parts of multiples of 8 rows, up to h/8 parts,
   * each a separate work item writing its own rows of C (no atomics, no workspace). */
  VBSR_PLAN_NO_SPLIT = 1u << 1,
  /* RHS 64 only, results identical either way: force the raw-B operand stacks (the pre-pass
   * writes raw B rows, the kernel forms their lo parts) or the pre-split ones (hi and lo rows
   * from the pre-pass). By default the plan picks raw-B when the pre-split stacks, K x 512
   * bytes, exceed 64 MB and would not stay in L2. */
  VBSR_PLAN_STACKS_RAW = 1u << 3,
  VBSR_PLAN_STACKS_PRESPLIT = 1u << 4,
  /* RHS 64 only, results identical: the SpMM reads the raw-B stack rows straight from B (16-byte
   * asynchronous copies of each column's run of values) instead of from a pre-pass buffer, so an
   * execute is one launch and the plan allocates no stack buffer. */
  VBSR_PLAN_B_DIRECT = 1u << 5,
  /* RHS <= 32, results within the same bound: block rows of height 8 or 16 (unless heavy) are
   * computed in plain fp32 on the CUDA cores by CTAs of the pre-pass launch instead of on the
   * tensor cores. The tensor-core kernel then gets shorter (headline: 75 -> 54 us), but the
   * pre-pass launch gets longer by more than that (its latency-bound CUDA-core rows run before the
   * SpMM), so it is off by default. */
  VBSR_PLAN_CUDA_CORE_ROWS = 1u << 6,
  /* Results identical: B's operand stacks are formed by the SpMM's own CTAs before their
   * pipelines start (a grid-wide arrival count in device memory, bounded waits), so an execute is
   * one launch instead of the pre-pass launch plus the SpMM. Off by default: it is slower (headline
   * 92 against 85 us, large config 15.8 against 14.5 ms), because the SpMM's pipelines cannot start
   * before every CTA's share of the stacks is done, while the separate pre-pass already overlaps
   * the SpMM's prologue (programmatic dependent launch). The CTAs wait for one another, so they
   * must all be resident (one per SM, at most one per SM of the device); a concurrent kernel that
   * holds SMs for longer than the plan's wait limit makes the execute report VBSR_TIMEOUT. */
  VBSR_PLAN_FUSED_PREPASS = 1u << 7,
  /* Diagnostics for performance analysis only; C is WRONG with either flag set: */
  VBSR_PLAN_DIAG_SKIP_COPIES = 1u << 8, /* producers arm the stages without copying any data  */
  VBSR_PLAN_DIAG_SKIP_MATH = 1u << 9,   /* consumers wait for the data but compute nothing     */
  /* Timing only: skip the B pre-pass and reuse the operand stacks the previous execute of this
   * plan formed; C is correct only if B is unchanged since then. */
  VBSR_PLAN_DIAG_SKIP_PREPASS = 1u << 10
};

/* Plan::Plan (plan.cpp:5-18): rhs must be 8, 16, 32 or 64. The plan schedules the block rows
 * of `m` once (per-SM work lists balanced by a byte cost model, heavy block rows cut into row
 * parts, pipeline stages of 8-column groups), uploads that schedule to the matrix's device and allocates the buffer the B pre-pass
 * writes (K/8 tiles of B's hi and lo rows); the matrix must outlive the plan. */
vbsr_status vbsr_plan_create(const vbsr_matrix* m, int rhs, int kernel, vbsr_plan** out);
vbsr_status vbsr_plan_create_ex(const vbsr_matrix* m, int rhs, int kernel, uint32_t flags,
                                vbsr_plan** out);
vbsr_status vbsr_plan_destroy(vbsr_plan* p);

/* Plan::execute (plan.cpp:19-22): enqueues C = A * B on `stream` (two kernels: the B pre-pass
 * into the plan's buffer, then the SpMM) and returns. B is K x rhs and C is M x rhs, column-major
 * device buffers on the matrix's device. C is fully overwritten (rows with no blocks become 0). No
 * allocation, no host synchronisation. Concurrent calls on one plan from several host threads or
 * streams are safe, with any B and C: the executes of one plan share its pre-pass buffer, so each
 * one is ordered on the GPU after the plan's previous execute, whatever stream that used (an event
 * the plan records; the host never waits). Inside a CUDA stream capture that cross-stream ordering
 * is not added: executes captured on one stream are ordered by it, executes captured on several
 * streams must be ordered by the graph's own dependencies. Launch failures return VBSR_CUDA_ERROR
 * (cudaGetLastError right after the launch). */
vbsr_status vbsr_plan_execute(const vbsr_plan* p, const float* B, float* C, vbsr_stream_t stream);

/* Same computation as vbsr_plan_execute, for callers that must not have device memory allocated
 * on their behalf (hosts that own every device allocation, or paths where the implicit device
 * synchronisation of cudaMalloc/cudaFree is not allowed). No reference counterpart: the reference
 * has no such entry point. It calls no cudaMalloc, cudaFree or other allocating routine; the
 * kernel's status words and per-CTA timestamps live instead in one fixed array compiled into the
 * library (16 KB per GPU, kept until the process exits), and plans of more than 1024 CTAs are
 * rejected with VBSR_INVALID_ARGUMENT. The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress); make that first call before any stream capture. Each call clears
 * the array's used part first, and all calls share it, so calls that overlap on the GPU race on it
 * (their C results are unaffected, only the reported status/timestamps). With cta_times == NULL the
 * call is asynchronous like vbsr_plan_execute and reports no kernel-side error: a VBSR_TIMEOUT or
 * VBSR_BOUNDS_VIOLATION recorded by that launch is overwritten by the next call's clearing, so a
 * caller that needs the kernel's status uses the reporting form. With cta_times != NULL the call
 * synchronises `stream`, copies up to cta_times_len timestamps ((start, end) pairs in ns, per CTA)
 * and returns VBSR_TIMEOUT, VBSR_BOUNDS_VIOLATION or (any other nonzero status word)
 * VBSR_CUDA_ERROR if the kernel recorded one. B or C not 16-byte aligned take a plain row kernel
 * that records neither status nor timestamps: the reporting form then waits for it and returns
 * zeros in cta_times. */
vbsr_status vbsr_plan_execute_noalloc(const vbsr_plan* p, const float* B, float* C,
                                      vbsr_stream_t stream, uint64_t* cta_times,
                                      int cta_times_len);

/* Plan::launch_count (plan.cpp:23-31): kernel launches per execute (2 here: the B pre-pass and
 * the SpMM kernel). */
vbsr_status vbsr_plan_launch_count(const vbsr_plan* p, int* out);

/* Reads and clears the plan's device status word (no reference counterpart): synchronises
 * `stream`, then returns VBSR_OK, VBSR_TIMEOUT or VBSR_BOUNDS_VIOLATION for the executions
 * enqueued since the last check. */
vbsr_status vbsr_plan_check_status(const vbsr_plan* p, vbsr_stream_t stream);

/* Human-readable schedule summary: RHS, items, pipeline stages, CTAs, ring depth, shared memory
 * per CTA and the kernel form. */
vbsr_status vbsr_plan_describe(const vbsr_plan* p, char* buf, size_t buf_len);

/* Test hook (no reference counterpart): makes the next executions stall one pipeline stage on
 * purpose (the producer withholds one stage and issues no copy for it) and caps every in-kernel
 * wait at `wait_limit_cycles` SM clocks, so that the timeout path can be exercised without
 * hanging the GPU. drop_stage < 0 switches the hook off. */
vbsr_status vbsr_plan_set_debug(vbsr_plan* p, int drop_stage, int64_t wait_limit_cycles);

/* Per-CTA timing (no reference counterpart; a tuning aid): enable != 0 makes the following
 * executions record, for every CTA, its start and end on the GPU's global nanosecond timer.
 * If `out` is not NULL, synchronises `stream` and copies up to out_len values (start, end pairs in
 * CTA order) from the last timed execution; values past the first 2 * tasks are 16 per-CTA cycle
 * counters that only an instrumented development build fills, zero otherwise. */
vbsr_status vbsr_plan_cta_timing(vbsr_plan* p, int enable, uint64_t* out, int out_len,
                                 vbsr_stream_t stream);
/* Per-task schedule facts (a tuning aid): team size in warps and the planner's cost estimate of
 * the task's most loaded team, for the first n tasks. Either output may be NULL. */
vbsr_status vbsr_plan_task_stats(const vbsr_plan* p, int32_t* team_warps, double* model_cost,
                                 int n);
/* How a plan divides the matrix's work (no reference counterpart; for reports and tests):
 * block rows on the tensor-core kernel (work items, of which split_rows were cut into row parts)
 * and on the CUDA-core path of the pre-pass launch, with their A value counts. */
typedef struct vbsr_plan_work {
  int64_t tc_items, tc_rows, split_rows, tc_values;
  int64_t cc_rows, cc_values, cc_scalar_rows;
} vbsr_plan_work;
vbsr_status vbsr_plan_work_info(const vbsr_plan* p, vbsr_plan_work* out);
/* Number of CTAs (tasks) one execution launches. */
vbsr_status vbsr_plan_num_tasks(const vbsr_plan* p, int* out);

/* ---- Raw launchers kept for source compatibility ------------------------------------------ */

/* launch_row_owned (row_owned.cu:397-423): C = A * B from a device view alone (no plan), one
 * CTA per block row, register-tiled. The unused reference arguments (row_shape_order and the
 * small/large counts) are accepted and ignored. */
vbsr_status vbsr_launch_row_owned(const vbsr_device_matrix* a, const int32_t* row_shape_order,
                                  int small_row_count, int large_row_count, const float* B,
                                  float* C, int rhs, vbsr_stream_t stream);
/* launch_row_owned_scalar (row_owned.cu:376-395): one output element per thread. */
vbsr_status vbsr_launch_row_owned_scalar(const vbsr_device_matrix* a, const float* B, float* C,
                                         int rhs, vbsr_stream_t stream);

/* ---- Input generation --------------------------------------------------------------------- */

enum {
  VBSR_DIST_UNIFORM = 0,
  VBSR_DIST_LOW_VARIANCE = 1,
  VBSR_DIST_HIGH_VARIANCE = 2,
  VBSR_DIST_BIMODAL = 3
};

/* PROFILE_REFERENCE reproduces generate() of the reference bit for bit (generator.cpp:7-88:
 * its size tables, cyclic +-degree local window, std::mt19937_64 draw order and
 * std::uniform_real_distribution<float>(-1,1) values). PROFILE_SPEC implements the block-size
 * distributions and clamped local window of the benchmark specification, draws structure from
 * std::mt19937_64(seed) and fills values with the counter-based generator, so any slice of the
 * values can be regenerated independently (in parallel, or on the device). */
enum { VBSR_PROFILE_REFERENCE = 0, VBSR_PROFILE_SPEC = 1 };

typedef struct vbsr_generator_options {
  int32_t block_rows, block_cols, degree;
  int32_t rhs_width;    /* carried for parity with GeneratorOptions; unused */
  int32_t distribution; /* VBSR_DIST_* */
  int32_t local_columns;
  uint64_t seed;
  int32_t profile;      /* VBSR_PROFILE_* */
  int32_t with_values;  /* 0: structure only (values empty; PROFILE_SPEC only) */
  int32_t threads;      /* host threads for value generation (<= 0: all cores) */
} vbsr_generator_options;

typedef struct vbsr_host_matrix vbsr_host_matrix; /* owning host matrix (HostMatrix) */

/* generate() (generator.cpp:7-88). Invalid dimensions give VBSR_INVALID_ARGUMENT with the
 * reference's message. */
vbsr_status vbsr_generate(const vbsr_generator_options* opts, vbsr_host_matrix** out);
vbsr_status vbsr_host_matrix_view_get(const vbsr_host_matrix* h, vbsr_host_matrix_view* out);
vbsr_status vbsr_host_matrix_free(vbsr_host_matrix* h);

/* ---- Real matrices: CSR conversion and the on-disk format -------------------------------- */

/* No reference counterpart: the reference has no loader or file format. Converts a scalar CSR
 * matrix (rows x cols; row_ptr has rows + 1 entries, col_idx / values row_ptr[rows]) into the VBSR
 * host format for the given block partition (row_sizes sum to rows, col_sizes to cols; every size
 * a multiple of 8 in [8, 64]): every block containing a nonzero becomes a dense block, zeros
 * elsewhere, duplicates summed. */
vbsr_status vbsr_host_matrix_from_csr(int64_t rows, int64_t cols, const int64_t* row_ptr,
                                      const int64_t* col_idx, const float* values,
                                      int32_t block_rows, const int32_t* row_sizes,
                                      int32_t block_cols, const int32_t* col_sizes,
                                      vbsr_host_matrix** out);
/* Binary VBSR file (magic "VBSRMAT1", then the HostMatrix arrays; layout in vbsr_io.cpp). Save
 * validates the matrix first; load validates what it read. */
vbsr_status vbsr_host_matrix_save(const vbsr_host_matrix_view* host, const char* path);
vbsr_status vbsr_host_matrix_load(const char* path, vbsr_host_matrix** out);

/* Counter-based U[-1,1) generator: out[i] = f(seed, stream, first + i). Used for PROFILE_SPEC
 * values (stream VBSR_STREAM_VALUES) and dense panels (VBSR_STREAM_DENSE). Host version; the
 * device version below gives bit-identical floats. */
enum { VBSR_STREAM_VALUES = 0xA11CE, VBSR_STREAM_DENSE = 0xB0B };
vbsr_status vbsr_fill_uniform(uint64_t seed, uint64_t stream, uint64_t first, uint64_t count,
                              float* out, int threads);
vbsr_status vbsr_fill_uniform_device(uint64_t seed, uint64_t stream, uint64_t first,
                                     uint64_t count, float* out_device, vbsr_stream_t cuda_stream);

/* std::mt19937(seed) + std::uniform_real_distribution<float>(-1,1), the dense input the
 * reference's tests draw (tests/test_main.cpp:42-51). */
vbsr_status vbsr_fill_mt19937(uint32_t seed, uint64_t count, float* out);

/* ---- Multi-GPU block-row partition -------------------------------------------------------- */

/* Splits the block rows into `parts` contiguous ranges of balanced cost (no reference
 * counterpart). Cost of a row = 4 * its value count + 4 * rhs * (sum of its block widths), i.e.
 * the A bytes it streams plus the B bytes it stages. bounds[0..parts] receives the range
 * boundaries (bounds[0] = 0, bounds[parts] = block_rows). */
vbsr_status vbsr_partition_rows(const vbsr_host_matrix_view* host, int parts, int rhs,
                                int32_t* bounds);

/* ---- Multi-GPU plan (one process, several GPUs) ------------------------------------------- */

/* No reference counterpart (the reference is single-GPU). A multi-GPU plan partitions the block
 * rows of a host matrix into `ngpus` contiguous ranges of balanced cost (vbsr_partition_rows),
 * builds each range's shard matrix and plan on devices[r] (devices may repeat), and owns per
 * shard a full K x rhs replica of B, a C block of the shard's c_rows x rhs (ld c_rows) and a
 * stream. Execute runs every shard's plan on its own stream: no reduction, no exchange, no NCCL.
 * kernel and flags are those of vbsr_plan_create_ex. */
typedef struct vbsr_multi_plan vbsr_multi_plan;
typedef struct vbsr_multi_shard {
  int32_t device;
  int32_t row_begin, row_end; /* block rows of the shard                                   */
  int64_t c_row0, c_rows;     /* its rows of C: [c_row0, c_row0 + c_rows) of the M rows     */
  float* B;                   /* device pointer: the shard's B replica (K x rhs, ld K)      */
  float* C;                   /* device pointer: the shard's C block (c_rows x rhs, ld c_rows) */
  vbsr_plan* plan;            /* the shard's plan (owned by the multi-plan)                 */
  vbsr_stream_t stream;       /* the shard's stream (owned by the multi-plan)               */
} vbsr_multi_shard;

vbsr_status vbsr_multi_plan_create(const vbsr_host_matrix_view* host, int ngpus,
                                   const int* devices, int rhs, int kernel, uint32_t flags,
                                   vbsr_multi_plan** out);
/* Like vbsr_multi_plan_create, with the values generated on each device from `seed` (as in
 * vbsr_matrix_create_rows_generated); host->values may be NULL. */
vbsr_status vbsr_multi_plan_create_generated(const vbsr_host_matrix_view* host, int ngpus,
                                             const int* devices, int rhs, int kernel,
                                             uint32_t flags, uint64_t seed,
                                             vbsr_multi_plan** out);
vbsr_status vbsr_multi_plan_destroy(vbsr_multi_plan* mp);
vbsr_status vbsr_multi_plan_count(const vbsr_multi_plan* mp, int* ngpus);
vbsr_status vbsr_multi_plan_shard(const vbsr_multi_plan* mp, int rank, vbsr_multi_shard* out);
/* Copies B (K x rhs, column-major) into every shard's replica: first into shard 0 from `B`
 * (host memory if src_device < 0, else device memory on src_device), then peer to peer along a
 * doubling tree (in round t shards [0, 2^t) each copy their replica to shard i + 2^t), so N
 * replicas take ceil(log2 N) rounds over NVLink. Asynchronous on the shards' streams: `B` must
 * be complete when the call is made and stay valid until the next synchronize. */
vbsr_status vbsr_multi_plan_replicate_B(vbsr_multi_plan* mp, const float* B, int src_device);
/* Enqueues every shard's execute on its stream (replica B, shard C), bracketed by events. */
vbsr_status vbsr_multi_plan_execute(vbsr_multi_plan* mp);
/* Waits for every shard, checks each plan's status word, and gives the longest shard time of
 * the last execute in ms (device events; max over shards). max_ms may be NULL. */
vbsr_status vbsr_multi_plan_synchronize(vbsr_multi_plan* mp, float* max_ms);
/* Assembles C (M x rhs, column-major, ld M) from the shards: host memory if dst_device < 0,
 * else device memory on dst_device (shards on other devices copy peer to peer). Returns when
 * the copies are done. */
vbsr_status vbsr_multi_plan_gather_C(vbsr_multi_plan* mp, float* C, int dst_device);

/* ---- Buffers shared between processes (one process per GPU) ------------------------------ */

/* No reference counterpart (the reference is single-GPU). For the one-process-per-GPU layout: each
 * rank allocates its B replica with vbsr_shared_buffer_create, exchanges the handle from
 * vbsr_shared_buffer_export with the other ranks (any host channel), maps theirs with
 * vbsr_shared_buffer_open, and fills its replica by copy-engine peer copies over NVLink
 * (vbsr_copy_async, one cudaMemcpyAsync per chunk) with no NCCL involved. A mapped peer buffer is
 * read-only by convention and must be closed (vbsr_shared_buffer_close) before its owner destroys
 * it. Ordering between processes is the caller's (a host barrier after each copy phase). */
typedef struct vbsr_shared_buffer vbsr_shared_buffer;
typedef struct vbsr_ipc_handle {
  unsigned char bytes[64];
} vbsr_ipc_handle;
vbsr_status vbsr_shared_buffer_create(int device, int64_t bytes, vbsr_shared_buffer** out);
vbsr_status vbsr_shared_buffer_destroy(vbsr_shared_buffer* b);
vbsr_status vbsr_shared_buffer_ptr(const vbsr_shared_buffer* b, void** ptr);
vbsr_status vbsr_shared_buffer_export(const vbsr_shared_buffer* b, vbsr_ipc_handle* out);
vbsr_status vbsr_shared_buffer_open(const vbsr_ipc_handle* handle, int device, void** peer_ptr);
vbsr_status vbsr_shared_buffer_close(void* peer_ptr, int device);
/* cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, stream): host, device or mapped peer memory
 * on either side. */
vbsr_status vbsr_copy_async(void* dst, const void* src, int64_t bytes, vbsr_stream_t stream);

/* Byte counts of the benchmark's roofline: the compulsory bytes of the reference VBSR format,
 * 4*sum(h*w) + 4*nnzb + 8*(nnzb+1) + 4*(R+1) + 4*R + 8*(R+1) + 4*S + 8*(S+1) + 4*K*N + 4*M*N,
 * and the useful flops 2*sum(h*w)*N, for block rows [row_begin, row_end) (the full column
 * structure and full B are counted). */
vbsr_status vbsr_compulsory_bytes(const vbsr_host_matrix_view* host, int32_t row_begin,
                                  int32_t row_end, int rhs, double* bytes, double* flops);

#ifdef __cplusplus
}
#endif
#endif /* VBSR_B200_H */
