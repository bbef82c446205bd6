/*
 * sf_q4.h -- C ABI of the B200 (sm_100a) Q4Linear kernels.
 *
 * This is the drop-in boundary for siliconfer's int4 weight-only linear path.
 * Every pointer is a DEVICE pointer (cudaMalloc / torch CUDA storage) unless a
 * comment says otherwise, and every call is asynchronous on `stream`
 * (a cudaStream_t passed as void*; NULL = legacy default stream).  The caller
 * owns every buffer, as in the reference's C kernels
 * (siliconfer/kernels/neon/q4_gemv.h:17-62).  Shape errors are reported as a
 * status code instead of the reference binding's std::runtime_error
 * (siliconfer/kernels/neon/bindings.cpp:24-40, 98-140); sf_last_error() gives
 * the same message text.
 *
 * Storage format (unchanged from the reference, q4_gemv.h:5-12 and
 * siliconfer/kernels/neon/__init__.py:42-81):
 *   W       uint8 [N, K/2]  byte j of row i = w(i,2j) | w(i,2j+1) << 4
 *                           sym: two's-complement nibbles (-8..7)
 *                           asym: unsigned nibbles (0..15)
 *   scales  float [N, K/group_size]
 *   zeros   float [N, K/group_size] or NULL (NULL selects the symmetric layout)
 *   x / X   [T, K] row-major, dtype SF_F32 / SF_F16 / SF_BF16
 *   y / Y   [T, N] row-major, dtype SF_F32 / SF_F16 / SF_BF16
 */
#ifndef SF_Q4_H_
#define SF_Q4_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  SF_OK = 0,
  SF_ERR_NULL = 1,        /* a required pointer is NULL                       */
  SF_ERR_SHAPE = 2,       /* N/K/T/group_size inconsistent                     */
  SF_ERR_DTYPE = 3,       /* unknown dtype code                                */
  SF_ERR_ALIGN = 4,       /* pointer alignment the kernel needs is not met     */
  SF_ERR_CUDA = 5,        /* a CUDA runtime call failed                        */
  SF_ERR_UNSUPPORTED = 6, /* valid request this build does not implement       */
  SF_ERR_TIMEOUT = 7,     /* a device-side bounded wait expired                */
  SF_ERR_COMM = 8,        /* tensor-parallel peer exchange failed              */
  SF_ERR_CAPTURE = 9      /* library scratch must grow while the stream is being
                             captured: run the same shape once on that stream
                             before capturing                                  */
} sf_status;

typedef enum { SF_F32 = 0, SF_F16 = 1, SF_BF16 = 2 } sf_dtype;

/* Human-readable text of a status code, and the detailed message of the last
   failing call on this host thread (mirrors bindings.cpp:27-39 wording). */
const char* sf_status_string(int status);
const char* sf_last_error(void);
int sf_version(void);

/* ---- reference-named entry points (fp32 activations in and out) ----------
 * Each replaces the reference C function of the same role:
 *   sf_q4_gemv_sym   <- q4_gemv_sym_neon   (q4_gemv.h:17-24;  bindings.cpp:45-55)
 *   sf_q4_gemv_scalar<- q4_gemv_sym_scalar (q4_gemv.h:27-33;  bindings.cpp:60-70)
 *   sf_q4_gemv_asym  <- q4_gemv_asym_neon  (q4_gemv.h:36-43;  bindings.cpp:75-92)
 *   sf_q4_gemm_sym   <- q4_gemm_sym_neon   (q4_gemv.h:46-53;  bindings.cpp:97-119)
 *   sf_q4_gemm_asym  <- q4_gemm_asym_neon  (q4_gemv.h:56-62;  bindings.cpp:124-150)
 * Argument order and meaning follow the reference; `stream` is appended.    */
int sf_q4_gemv_sym(const uint8_t* W, const float* scales, const float* x, float* y,
                   int out_f, int in_f, int group_size, void* stream);
int sf_q4_gemv_scalar(const uint8_t* W, const float* scales, const float* x, float* y,
                      int out_f, int in_f, int group_size, void* stream);
int sf_q4_gemv_asym(const uint8_t* W, const float* scales, const float* zeros,
                    const float* x, float* y, int out_f, int in_f, int group_size,
                    void* stream);
int sf_q4_gemm_sym(const uint8_t* W, const float* scales, const float* X, float* Y,
                   int out_f, int in_f, int T, int group_size, void* stream);
int sf_q4_gemm_asym(const uint8_t* W, const float* scales, const float* zeros,
                    const float* X, float* Y, int out_f, int in_f, int T,
                    int group_size, void* stream);

/* ---- general entry point used by Q4Linear ----------------------------------
 * Y[T,N] = X[T,K] @ dequant(W)^T (+ bias), fp32 accumulation.
 * Replaces Q4Linear.__call__'s kernel dispatch (siliconfer/model/q4_linear.py:
 * 57-66): zeros != NULL selects the asymmetric kernel, bias (fp32 [N], may be
 * NULL) is added after the product.  T <= 16 (T <= 8 at group size 32) runs
 * the decode GEMV kernel in one pass over W (above 8 tokens on a two-digit
 * activation grid: rounding at most 2^-15 of each group's max |x|); T >= 48
 * runs the prefill GEMM; in between, the decode kernel runs on chunks of 8
 * tokens.  flags: bit 0 = allow programmatic
 * dependent launch (the kernel may start streaming weights before the
 * previous kernel on `stream` has finished; x is read only after it has). */
int sf_q4_linear(const uint8_t* W, const float* scales, const float* zeros,
                 const float* bias, const void* X, int x_dtype, void* Y, int y_dtype,
                 int N, int K, int T, int group_size, int flags, void* stream);
#define SF_FLAG_PDL 1

/* ---- a decode step: many GEMVs in one persistent launch -------------------
 * The reference calls Q4Linear once per projection, seven times per layer
 * (siliconfer/model/layers.py:93-95, 133, 144; q4_linear.py:49-68).  Here a
 * caller describes the whole sequence once and replays it: one cooperative
 * launch streams every task's weights back to back, so HBM stays busy across
 * projection boundaries.
 * Ordering: a task with wait_before != 0 starts a new phase.  Every task of a
 * phase reads its X only after all tasks of the previous phase have written
 * their Y (bounded device-side waits on per-task completion counters), which
 * is how o_proj <- attention(q, k, v) is expressed.  Tasks of one phase run
 * concurrently.  Only the first phase's X must exist before the launch.
 * All tasks must share T (1..16; 1..8 at group size 32), the layout (zeros NULL or not) and the group
 * class (group_size % 128, % 64 or % 32 == 0); group_size a power of two in
 * 32..256, K % 32 == 0, W/scales/zeros/X 16-byte aligned.  `workspace` is
 * caller-owned device memory of sf_q4_step_workspace_bytes(tasks, ntasks)
 * bytes, 256-byte aligned, kept alive until sf_q4_step_destroy; it holds the
 * task table, the completion counters and the activations in integer form, so
 * two handles that run concurrently need two workspaces.
 * create() uploads the table synchronously; run() is asynchronous. */
typedef struct {
  const uint8_t* W;
  const float* scales;
  const float* zeros;   /* NULL: symmetric */
  const float* bias;    /* NULL: none */
  const void* X;        /* [T, K] of x_dtype */
  void* Y;              /* [T, N] of y_dtype */
  int N, K, T, group_size, x_dtype, y_dtype, wait_before;
  int epilogue;         /* 0, or SF_EPI_SWIGLU (see sf_q4_linear_swiglu; N = gate + up rows) */
  int bits;             /* weight bit width: 0 or 4 (packed [N, K/2]), 2 (packed [N, K/4], see
                           sf_q2_linear); every task of a step has the same */
} sf_q4_task;
#define SF_EPI_SWIGLU 1
size_t sf_q4_step_workspace_bytes(const sf_q4_task* tasks, int ntasks);
int sf_q4_step_create(const sf_q4_task* tasks, int ntasks, void* workspace, size_t workspace_bytes,
                      void** handle_out);
int sf_q4_step_run(void* handle, void* stream);
void sf_q4_step_destroy(void* handle);

/* ---- 2-bit weights ------------------------------------------------------
 * The reference quantizes to 2 bits (siliconfer/quant/primitives.py:154-245,
 * quantize_sym_int2 / quantize_asym_int2) and packs four values per byte
 * (pack_int2, primitives.py:383-404: element i in bits 2i..2i+1), but its
 * loader refuses to serve them (siliconfer/engine/q4_loader.py:142-154: no
 * int2 kernel).  This is that kernel: W uint8 [N, K/4]; symmetric q in
 * [-2, 1] (two's complement, zeros NULL) or asymmetric q in [0, 3] with fp32
 * zeros; y = X @ dequant(W)^T (+ bias), dequant (q - z) * s as in
 * dequantize_sym_int2 / dequantize_asym_int2 (primitives.py:184-245).
 * K % 64 == 0 and group_size 128 or 256; any T (the decode kernel: one
 * launch up to 16 tokens, chunks of 8 above). */
int sf_q2_linear(const uint8_t* W, const float* scales, const float* zeros, const float* bias,
                 const void* X, int x_dtype, void* Y, int y_dtype, int N, int K, int T,
                 int group_size, void* stream);

/* ---- MLP gate/up with the SwiGLU activation fused ------------------------
 * Replaces the gate/up half of siliconfer's MLP.__call__ (siliconfer/model/
 * layers.py:144: down_proj(silu(gate_proj(x)) * up_proj(x))): both
 * projections read x once, in one GEMV whose epilogue writes
 *   Y[T, N] = silu(X @ Wg^T + bg) * (X @ Wu^T + bu),  silu(v) = v / (1 + e^-v),
 * ready to be down_proj's input.  W, scales, zeros and bias hold the gate and
 * up triples INTERLEAVED in blocks of 16 rows: rows 32i .. 32i+15 are gate rows
 * 16i .. 16i+15, rows 32i+16 .. 32i+31 the same up rows (2N rows in all;
 * N % 16 == 0).  Decode sizes only (T <= 16, T <= 8 at group size 32; shape
 * rules of the decode kernel); other shapes return SF_ERR_UNSUPPORTED. */
int sf_q4_linear_swiglu(const uint8_t* W, const float* scales, const float* zeros,
                        const float* bias, const void* X, int x_dtype, void* Y, int y_dtype,
                        int N, int K, int T, int group_size, void* stream);
/* The same activation applied to an already computed product of the
 * interleaved rows: in [T, 2N] fp32 (the sf_q4_linear output of those rows,
 * bias not added), bias [2N] interleaved or NULL, out [T, N] of out_dtype. */
int sf_swiglu_interleaved(const float* in, void* out, int out_dtype, int T, int N, const float* bias,
                          void* stream);

/* sf_q4_linear for T <= 16 that allocates nothing.  No counterpart in the
 * reference (its kernels need no device scratch).  sf_q4_linear keeps a
 * library-owned scratch buffer per stream and grows it with cudaMalloc the
 * first time it sees a shape; this entry point is for callers that cannot let
 * a library allocate (a process that reserves the whole GPU for its own pool,
 * code where an allocation would stall or be refused).  It uses a fixed 4 MiB
 * buffer compiled into the library's device image instead:
 *   - limits: N <= 524288 rows, and the activation blocks (about
 *     3*T*K + 8*T*K/group_size bytes) must fit in 4032 KiB, e.g. T = 8 up to
 *     K = 160000 at group 128; larger requests fail with SF_ERR_SHAPE and a
 *     message naming the limit.  When the k-split partial sums would not fit,
 *     fewer k-splits are used.
 *   - the first call on each device looks the buffer up
 *     (cudaGetSymbolAddress); make that first call before any stream capture.
 *   - there is ONE buffer per device: calls that overlap in time on the same
 *     device (other streams, other host threads) race on it.  Order them,
 *     e.g. issue them all on one stream.
 * Same arguments, layouts and results as sf_q4_linear otherwise (no flags). */
int sf_q4_linear_static_scratch(const uint8_t* W, const float* scales, const float* zeros,
                                const float* bias, const void* X, int x_dtype, void* Y,
                                int y_dtype, int N, int K, int T, int group_size, void* stream);

/* ---- tensor parallelism across the GPUs of one node -----------------------
 * The reference has no parallel form of Q4Linear (siliconfer/model/
 * q4_linear.py:32-68 is single-device); these entry points replace the
 * row-parallel projections (o_proj, down_proj; siliconfer/model/layers.py:133,
 * 144) of a model sharded over P ranks, one process per GPU.  A
 * column-parallel projection (q/k/v/gate/up) needs no exchange: each rank calls
 * sf_q4_linear on its own block of rows.  A row-parallel rank owns a block of
 * whole groups along K and calls sf_q4_linear_allreduce, which runs the GEMV
 * into the rank's exchange buffer and sums the partials of all ranks over
 * NVLink peer memory (rank order: every rank gets bitwise the same Y).
 * Set-up (once per rank, collective):
 *   sf_tp_comm_init    allocates this rank's exchange buffer (flags, two
 *                      slots of slot_bytes, then arena_bytes for the
 *                      regions of fused step tasks, see
 *                      sf_q4_step_create_tp) and writes its CUDA IPC handle
 *                      (sf_tp_handle_bytes() bytes) to handle_out;
 *   (exchange the handles between ranks, e.g. torch.distributed all_gather)
 *   sf_tp_comm_connect opens every peer's buffer (handles: world x handle
 *                      bytes, in rank order).
 * Every rank must issue the same sequence of all-reduce calls.  Waits on
 * peers are bounded (about 2 s); on expiry the kernel returns early and
 * sf_q4_check_device_error() reports SF_ERR_TIMEOUT.  An expired wait
 * POISONS the communicator for good: the ranks' call epochs are out of step,
 * so the rank that gave up marks its buffer and every peer's flag.  A peer
 * that arrives late, and every later all-reduce or fused step on any rank,
 * then returns at once without summing anything, and
 * sf_q4_check_device_error() reports SF_ERR_COMM.  Destroy the communicator
 * and create it again (on every rank) to continue. */
size_t sf_tp_handle_bytes(void);
int sf_tp_comm_init(int rank, int world, size_t slot_bytes, size_t arena_bytes, void** comm_out,
                    void* handle_out);
int sf_tp_comm_connect(void* comm, const void* handles);
/* Y[count] = sum over ranks of partial (fp32, device, count floats; NULL =
   already in place) + bias[i % ncols]; out of out_dtype. */
int sf_tp_allreduce(void* comm, const float* partial, void* out, int out_dtype, const float* bias,
                    long long count, int ncols, void* stream);
/* Row-parallel Q4Linear shard: Y = allreduce(X[T,K_shard] @ dequant(W_shard)^T) + bias. */
int sf_q4_linear_allreduce(void* comm, const uint8_t* W, const float* scales, const float* zeros,
                           const float* bias, const void* X, int x_dtype, void* Y, int y_dtype,
                           int N, int K, int T, int group_size, void* stream);
void sf_tp_comm_destroy(void* comm);

/* A tensor-parallel decode step as ONE persistent launch, the all-reduces
 * fused into the GEMV kernel.  Same tasks as sf_q4_step_create plus a role
 * per task:
 *   SF_ROLE_GEMV        an ordinary GEMV (column-parallel projections);
 *   SF_ROLE_PUSH        a row-parallel shard: each finished 32-row tile of its
 *                       fp32 partial is stored into every rank's exchange
 *                       region over NVLink (peer stores), followed by a
 *                       per-tile flag; Y may be NULL;
 *   SF_ROLE_REDUCE + i  the all-reduce of earlier task i (a PUSH task of the
 *                       same N): waits (bounded) for every rank's flag of each
 *                       tile, sums the ranks in rank order (+ bias) and
 *                       writes Y of y_dtype.  Give it task i's W, scales,
 *                       zeros, X, K and group_size (unused) and its own Y,
 *                       bias and y_dtype.
 * Regions are carved from the communicator's arena at creation (the same
 * task lists on every rank give the same offsets), two parities per region
 * so that consecutive runs never overwrite data a peer is still reading.
 * Every rank must create the same step and run it the same number of times;
 * the launch is cooperative.  The workspace is sized by
 * sf_q4_step_workspace_bytes on the same task list. */
#define SF_ROLE_GEMV 0
#define SF_ROLE_PUSH 1
#define SF_ROLE_REDUCE 2
int sf_q4_step_create_tp(const sf_q4_task* tasks, const int* roles, int ntasks, void* comm,
                         void* workspace, size_t workspace_bytes, void** handle_out);

/* ---- decode attention over an int8-quantized KV cache --------------------
 * Replaces fused_quantized_attention_decode (siliconfer/kernels/metal/
 * q4_attention.py:200-260) over the cache of siliconfer/model/kv_cache.py:49-69:
 *   q        [B, H, D] of q_dtype (one decode token per sequence)
 *   k_codes  [B, Hkv, T, D] int8, k_scales [B, Hkv, T] fp32 (per-vector scale)
 *   v_codes, v_scales likewise
 *   out      [B, H, D] of out_dtype = softmax(q.k / sqrt(D)) . v, fp32 math.
 * H % Hkv == 0 (GQA; group sizes 1, 2, 4, 7, 8), D in {64, 128, 256}.
 * n_split <= 0 picks the T-split count (sf_kv_attention_splits); the
 * caller-owned workspace holds the splits' partial results and must have
 * sf_kv_attention_workspace_bytes(B, H, D, n_split) bytes. */
size_t sf_kv_attention_workspace_bytes(int B, int H, int D, int n_split);
int sf_kv_attention_splits(int B, int Hkv, int T);
int sf_kv_attention_decode(const void* q, int q_dtype, const int8_t* k_codes, const float* k_scales,
                           const int8_t* v_codes, const float* v_scales, void* out, int out_dtype,
                           int B, int H, int Hkv, int T, int D, int n_split, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Device dequant to fp32/fp16/bf16 [N, K].  fp32 output is bit-exact with
   dequantize_sym / dequantize_asym (siliconfer/quant/primitives.py:54-75,
   117-140); fp16/bf16 are that value rounded to nearest even. */
int sf_q4_dequant(const uint8_t* W, const float* scales, const float* zeros, void* out,
                  int out_dtype, int N, int K, int group_size, void* stream);

/* Device RTN quantize + pack of an fp32 [N, K] weight, bit-exact with
   pack_weights_sym / pack_weights_asym (siliconfer/kernels/neon/__init__.py:
   42-81 -> siliconfer/quant/primitives.py:24-51, 82-114).  zeros == NULL
   selects symmetric packing. */
int sf_q4_quantize_pack(const float* W, uint8_t* packed, float* scales, float* zeros,
                        int N, int K, int group_size, void* stream);

/* Sticky device-side error word (set when a bounded wait inside a kernel
   expires, or when a tensor-parallel kernel met a poisoned communicator).
   Synchronous: reads and clears it.  Returns SF_OK, SF_ERR_TIMEOUT, or
   SF_ERR_COMM (poisoned communicator; takes precedence). */
int sf_q4_check_device_error(void);

/* Number of kernels this library has launched since load (host counter). */
long long sf_q4_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif /* SF_Q4_H_ */
