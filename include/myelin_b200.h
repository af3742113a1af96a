/*
 * myelin_b200 C ABI — hand-written sm_100a kernels for the spiking-neuron hot
 * path of djsaunde/myelin: the fused-time LIF/ALIF membrane scan with its
 * reverse-time surrogate backward, and bit-packed spike pack/unpack/count.
 *
 * Conventions (every entry point):
 *   - Plain C: device pointers, sizes, scalars, and a cudaStream_t passed as
 *     `void*` (NULL = legacy default stream). No torch types.
 *   - Tensors are dense, C-contiguous, time-major [T, B, N] (state [B, N]),
 *     exactly the layout of the reference's Python API.
 *   - Return 0 on success; non-zero on error, with a message available from
 *     mb_last_error() (thread-local). Launch is asynchronous on `stream`.
 *   - Stateless and reentrant from any host thread; no allocation.
 *
 * The reference has no FFI: its boundary is a set of Python functions that
 * launch Triton kernels. Each entry point below cites the reference function
 * (path inside the reference project, file:line) whose work it replaces.
 */
#ifndef MYELIN_B200_H
#define MYELIN_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types of I/O tensors. */
enum mb_dtype {
  MB_F32 = 0,
  MB_BF16 = 1,
  MB_F16 = 2,
  MB_F64 = 3,
  MB_U8 = 4,  /* bool / uint8 / int8: nonzero byte = spike */
  MB_I16 = 5,
  MB_I32 = 6,
  MB_I64 = 7
};

/* Neuron models on the scan path. */
enum mb_neuron { MB_LIF = 0, MB_ALIF = 1 };

/* Izhikevich parameters, the fields and defaults of the reference's
 * IzhikevichParams (src/myelin/neurons.py:74-96); dt must be positive. */
typedef struct mb_izhikevich_params {
  float recovery_decay;       /* a, default 0.02 */
  float recovery_coupling;    /* b, default 0.2 */
  float reset_voltage;        /* default -65 */
  float recovery_jump;        /* default 8 */
  float threshold;            /* default 30 */
  float dt;                   /* default 1 */
  float voltage_square_coeff; /* default 0.04 */
  float voltage_coeff;        /* default 5 */
  float voltage_bias;         /* default 140 */
} mb_izhikevich_params;

/* Reset rule after a spike: HARD sets the membrane to `reset`
 * (src/myelin/neurons.py:113, functional.py:143); SUBTRACT removes the
 * (adaptive) threshold, m <- p - theta (extension, not in the reference). */
enum mb_reset { MB_RESET_HARD = 0, MB_RESET_SUBTRACT = 1 };

/* Surrogate derivative ids, numbered as src/myelin/triton/lif.py:356-370.
 * MB_SURR_NONE gives the exact gradient of the hard (non-surrogate) forward,
 * used by the plain lif_forward/alif_forward backward. */
enum mb_surrogate {
  MB_SURR_SIGMOID = 0,
  MB_SURR_FAST_SIGMOID = 1,
  MB_SURR_ATAN = 2,
  MB_SURR_TRIANGULAR = 3,
  MB_SURR_SUPERSPIKE = 4,
  MB_SURR_MULTI_GAUSSIAN = 5,
  MB_SURR_NONE = 6
};

/* Replay chunk (time steps) the backward uses: the forward writes one fp32
 * checkpoint of the state every MB_SCAN_CHUNK steps, the backward replays a
 * chunk in registers from it and walks it in reverse. */
#define MB_SCAN_CHUNK 16

/* Last error message of the calling host thread ("" if none). */
const char* mb_last_error(void);

/* Library version string. */
const char* mb_version(void);

/* Device status of every kernel with bounded waits (scan forward/backward, both
 * tensor-core GEMMs) on the current device: 0 = ok, 1 = a bounded wait for an
 * asynchronous copy or an MMA ran out (the kernel stopped early and its
 * outputs are incomplete). Synchronises the device. `clear` != 0 resets the
 * status to 0 after reading it. Returns -1 if the status can't be read.
 * No reference counterpart (the reference's Triton kernels never wait). */
int mb_device_status(int clear);

/* Code units whose status words mb_device_status combines. */
enum mb_unit { MB_UNIT_SCAN = 0, MB_UNIT_SCAN_FAST = 1, MB_UNIT_GEMM = 2 };

/* Diagnostic: launch one tiny kernel in `unit` whose single bounded wait
 * (budget `polls`, 1..65536) is on a barrier nothing arrives at, so it runs
 * out the way a stalled copy would: the kernel records status 1 (visible
 * through mb_device_status) and returns. It touches no memory but the status
 * word. Used by tests to show that a timeout is reported; no reference
 * counterpart. */
int mb_debug_wait_timeout(int unit, int polls, void* stream);

/* Number of chunk checkpoints for T steps: ceil(T / MB_SCAN_CHUNK). */
int64_t mb_scan_num_checkpoints(int64_t T);

/*
 * Fused-time forward scan over x[T,B,N] for LIF or ALIF neurons.
 *   p_t = m_{t-1} * decay + x_t            (two roundings, no FMA)
 *   theta_t = threshold [+ beta * a_{t-1}]  (ALIF)
 *   s_t = p_t >= theta_t
 *   m_t = s_t ? reset : p_t   (HARD)   |  s_t ? p_t - theta_t : p_t  (SUBTRACT)
 *   a_t = a_{t-1} * adapt_decay + s_t       (ALIF)
 * The membrane/adaptation are carried in fp32 whatever `dtype` is.
 * Inputs : x [T,B,N] (dtype), v0 [B,N] (dtype), a0 [B,N] (dtype, ALIF only).
 * Outputs (each may be NULL):
 *   vT, aT        final state [B,N] (dtype)
 *   spikes        dense 0/1 [T,B,N] (dtype)
 *   packed        int32 words [T,B,ceil(N/32)], bit j of word w = neuron 32w+j
 *   rates         spike count / T [B,N] (dtype)
 *   ckpt_v/ckpt_a fp32 state at the start of every MB_SCAN_CHUNK-step chunk,
 *                 [mb_scan_num_checkpoints(T), B, N], consumed by the backward.
 * Replaces: kernels.lif_forward (src/myelin/kernels.py:52) -> triton/lif.py:16-95;
 *   kernels.lif_forward_packed_spikes (kernels.py:96) -> triton/lif.py:98-192;
 *   kernels.alif_forward (kernels.py:159) -> triton/generated.py:1159-1189;
 *   surrogate forward of kernels.surrogate_lif_forward (kernels.py:249)
 *   -> triton/lif.py:195-222,373-405; rate forward (triton/lif.py:823-889).
 */
int mb_scan_forward(int neuron, int dtype, const void* x, const void* v0, const void* a0,
                    void* vT, void* aT, void* spikes, int32_t* packed, void* rates,
                    float* ckpt_v, float* ckpt_a, int64_t T, int64_t B, int64_t N,
                    float decay, float threshold, float reset, float adapt_decay,
                    float beta, int reset_mode, void* stream);

/*
 * Packed-only LIF/ALIF forward (as mb_scan_forward with only `packed`) whose
 * words also go to `num_peers` (0..7) peer slots: `peers` is a host array of
 * device pointers, each the start of this rank's [T, B, ceil(N/32)] slot in
 * another rank's gather buffer (mapped with mb_ipc_open). The scan writes
 * `packed` (this rank's slot of its own buffer); one kernel on the same
 * stream then stores the slot into every peer slot at once over NVLink. Like mb_pack_count_scatter it
 * does not wait for peers: the caller orders later reads of the gather
 * buffers after every rank's call.
 * Replaces: kernels.lif_forward_packed_spikes (src/myelin/kernels.py:96-156)
 *   followed by distributed.packed_spike_all_gather (distributed.py:63-80),
 *   the forward-only communication path of the packed linear module
 *   (kernels.py:705-776, modules.py:906-943).
 */
int mb_scan_forward_packed_scatter(int neuron, int dtype, const void* x, const void* v0,
                                   const void* a0, void* vT, void* aT, int32_t* packed,
                                   void* const* peers, int num_peers, int64_t T, int64_t B,
                                   int64_t N, float decay, float threshold, float reset,
                                   float adapt_decay, float beta, int reset_mode, void* stream);

/*
 * Reverse-time surrogate backward of mb_scan_forward. Replays each chunk from
 * its checkpoint in registers (bit-identical to the forward), then walks it in
 * reverse:
 *   d   = slope * surrogate'(slope * (p - theta))
 *   HARD:     Gs = gs + gm*(reset - p) [+ ga];  gp = gm*(1 - s) + Gs*d
 *   SUBTRACT: Gs = gs - gm*theta       [+ ga];  gp = gm + Gs*d
 *   ALIF: ga <- ga*adapt_decay - beta*(Gs*d [+ gm*s for SUBTRACT])
 *   grad_x_t = gp;  gm <- gp * decay
 * gs = grad_spikes[t] (if given) + grad_rates / T (if given).
 * Inputs : x, ckpt_v, ckpt_a (ALIF) from the forward; grad_spikes [T,B,N],
 *          grad_rates [B,N], grad_vT [B,N], grad_aT [B,N] (dtype; each may be NULL).
 * Outputs: grad_x [T,B,N] (dtype, required), grad_v0 / grad_a0 [B,N] (nullable).
 * Replaces: triton/lif.py:252-336,408-551 (surrogate LIF backward) and the
 *   torch autograd through functional.surrogate_alif_unroll (functional.py:149-189).
 */
int mb_scan_backward(int neuron, int dtype, const void* x, const float* ckpt_v,
                     const float* ckpt_a, const void* grad_spikes, const void* grad_rates,
                     const void* grad_vT, const void* grad_aT, void* grad_x, void* grad_v0,
                     void* grad_a0, int64_t T, int64_t B, int64_t N, float decay,
                     float threshold, float reset, float adapt_decay, float beta,
                     int reset_mode, int surrogate, float slope, void* stream);

/*
 * mb_scan_backward plus grad_sum (fp32 [B*N], 8-byte aligned, nullable): for
 * every neuron the sum over t of grad_x as stored (in the I/O type), from
 * the last step to the first, in fp32. The LIF backward kernel forms it as it
 * writes grad_x; other kinds and layouts sum grad_x over t afterwards. The
 * bias gradient of a stream-synapse layer is the column sum of grad_sum
 * viewed as [B, N] (mb_column_sums), instead of a pass over [T*B, N].
 * Replaces: the bias-gradient reduction of src/myelin/triton/lif.py:1232-1258
 *   (float atomics there; fixed order here).
 */
int mb_scan_backward_sum(int neuron, int dtype, const void* x, const float* ckpt_v,
                         const float* ckpt_a, const void* grad_spikes, const void* grad_rates,
                         const void* grad_vT, const void* grad_aT, void* grad_x, void* grad_v0,
                         void* grad_a0, float* grad_sum, int64_t T, int64_t B, int64_t N,
                         float decay, float threshold, float reset, float adapt_decay,
                         float beta, int reset_mode, int surrogate, float slope, void* stream);

/*
 * Fused-time Izhikevich forward over x[T,B,N] (dtype MB_F32/BF16/F16):
 *   dv  = ((c2 * v) * v + c1 * v) + bias - u + x_t     (one rounding per op)
 *   p_v = v + dt * dv;   p_u = u + dt * (a * (b * v - u))
 *   s_t = p_v >= threshold
 *   v = s_t ? reset_voltage : p_v;   u = s_t ? p_u + recovery_jump : p_u
 * Inputs: x, v0, u0 [B,N]. Outputs (each may be NULL): vT, uT [B,N] and dense
 * 0/1 spikes [T,B,N], all of dtype. fp32 state carry; bit-exact with the
 * reference's torch path for fp32. Forward only.
 * Replaces: kernels.izhikevich_forward (src/myelin/kernels.py:202-246) ->
 *   triton/generated.py:1192-1227 / functional.izhikevich_unroll
 *   (functional.py:81-112).
 */
int mb_izhikevich_forward(int dtype, const void* x, const void* v0, const void* u0, void* vT,
                          void* uT, void* spikes, int64_t T, int64_t B, int64_t N,
                          const mb_izhikevich_params* params, void* stream);

/*
 * Dense projection on the tcgen05 tensor cores:
 *   C[M, N] = A[M, K] * B[N, K]^T (+ bias[N])
 * A, B: `in_dtype` (MB_BF16 or MB_F16), rows of K contiguous elements with
 * leading dimensions lda, ldb (multiples of 8, 16-byte aligned bases);
 * fp32 accumulation; C: `out_dtype` (MB_F32 or in_dtype), leading dimension
 * ldc; bias: optional, MB_F32/MB_BF16/MB_F16. Used for the stream synapse's
 * currents x[T*B, F] * W^T and its input gradient G[T*B, N] * W.
 * Replaces: the per-timestep tl.dot of src/myelin/triton/lif.py:554-612 and
 *   the projections of src/myelin/autograd.py:445-556 (torch.matmul).
 */
int mb_gemm_tn(int in_dtype, const void* A, int64_t lda, const void* B, int64_t ldb,
               const void* bias, int bias_dtype, int out_dtype, void* C, int64_t ldc, int64_t M,
               int64_t N, int64_t K, void* stream);

/* Operand layouts of mb_gemm. K-major: element (r, k) at r * ld + k (rows of K
 * contiguous elements). MN-major: element (r, k) at k * ld + r (K rows of M or
 * N contiguous elements), e.g. x[T*B, F] read as the M-major A of x^T. */
enum mb_major { MB_KMAJOR = 0, MB_MNMAJOR = 1 };

/*
 * General tensor-core GEMM (mb_gemm_tn is the K-major/K-major case):
 *   C[M, N] = sum over (i, j) of A_i[M, K] * B_j[N, K]^T (+ bias[N])
 * A_i / B_j: part i / j of A / B (`a_parts`, `b_parts` in 1..3, parts
 * `*_part_stride` elements apart, multiples of 8), each K-major or MN-major
 * (`a_major`, `b_major`; an M-major A needs an N-major B). The products kept
 * are those with i + j <= 2: with an fp32 operand split into 3 bf16 parts
 * (mb_split_bf16, part p holding the bits 8p below the leading ones) this is
 * the fp32 product to within 2^-24 relative per term, computed on the 16-bit
 * tensor cores with fp32 accumulation (bf16x6 for two split operands, x3 when
 * one side is exact in one part, e.g. 0/1 spikes). `a_nonzero` / `b_nonzero`
 * (device int per part, nullable, as written by mb_split_bf16) skip the
 * products of an all-zero part on the device. Leading dimensions: multiples
 * of 8; K-major also needs K % 8 == 0 and ld >= K; MN-major ld >= M (or N).
 * Bases 16-byte aligned. Out-of-range elements of the tiles read as zero.
 * K is accumulated in slices, each into an fp32 partial in `workspace`
 * (mb_gemm_workspace_bytes; nullable when that is 0) and the slices are then
 * summed in order in fp32 (+ bias): deterministic. Slices are used for fp32
 * output from split operands (at most 2048 of K each: the tensor cores' fp32
 * accumulation of one MMA is not correctly rounded, so its error grows with
 * the MMAs summed into one accumulator), and to occupy the SMs when the
 * output has few tiles and K is long (the weight gradient of a small or
 * narrow layer, K = T*B). With K >= 8192 and more 256 x 256 tiles than SM
 * pairs, only the tiles of the last, partial wave are sliced (their fp32
 * partials cover just their rows of C); the others are written directly.
 * Without the workspace these optional slices are skipped (same result up
 * to summation order).
 * Used for the stream synapse's currents x[T*B, F] * W[F, N] (B = W N-major,
 * no transposed copy), input gradient G * W^T (both K-major) and weight
 * gradient x^T G (A = x M-major, B = G N-major; no transposes).
 * Replaces: the tl.dot contractions of src/myelin/triton/lif.py:554-612 (forward),
 *   :1136-1180 (input gradient) and :1183-1228 (weight gradient), and the
 *   torch.matmul projections of src/myelin/autograd.py:445-556.
 */
int mb_gemm(int in_dtype, const void* A, int a_major, int64_t lda, int64_t a_part_stride,
            int a_parts, const int32_t* a_nonzero, const void* B, int b_major, int64_t ldb,
            int64_t b_part_stride, int b_parts, const int32_t* b_nonzero, const void* bias,
            int bias_dtype, int out_dtype, void* C, int64_t ldc, int64_t M, int64_t N, int64_t K,
            void* workspace, int64_t workspace_bytes, void* stream);

/* Workspace (bytes) mb_gemm needs for these sizes, part counts and output type
 * on the current device (0 when K is not sliced). */
int64_t mb_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int a_parts, int b_parts,
                                int out_dtype);

/*
 * Split src[rows, cols] (element (r, c) at r * src_row_stride + c *
 * src_col_stride, in elements; MB_F32, MB_BF16 or MB_F16) into `parts` (1..3)
 * bf16 matrices dst + p * dst_part_stride, element (r, c) at r * dst_ld + c,
 * whose sum is the fp32 source value exactly (part p = the bf16 rounding of
 * what parts 0..p-1 left; non-finite values stay in part 0). A 16-bit source
 * takes one part and keeps its own type: a plain re-laid-out copy (a
 * transposed view, or rows padded to 16 bytes). The destination region
 * [dst_rows, dst_cols] (at least the source's) is written in full, zeros
 * outside the source. `nonzero` (nullable, `parts` ints) is set to 1 for each
 * part holding a nonzero element, for mb_gemm's a_nonzero / b_nonzero.
 * No reference counterpart (operand preparation for mb_gemm).
 */
int mb_split_bf16(int src_dtype, const void* src, int64_t rows, int64_t cols,
                  int64_t src_row_stride, int64_t src_col_stride, int parts, void* dst,
                  int64_t dst_rows, int64_t dst_cols, int64_t dst_ld, int64_t dst_part_stride,
                  int32_t* nonzero, void* stream);

/*
 * fp32 product with a short contraction: C[M, N] = A[M, K] * B[N, K]^T, K <= 32,
 * both operands K-major (leading dimensions lda, ldb), fp32 FMAs with k in
 * order. For the input gradient of a narrow fp32 layer (G[T*B, 10] * W^T),
 * where tensor-core tiles would be mostly padding.
 * Replaces: src/myelin/triton/lif.py:1136-1180 (input gradient) for narrow layers.
 */
int mb_gemm_small_k(const float* A, int64_t lda, const float* B, int64_t ldb, float* C,
                    int64_t ldc, int64_t M, int64_t N, int64_t K, void* stream);

/* Workspace (bytes) mb_column_sums needs for a [rows, cols] source. */
int64_t mb_column_sums_workspace_bytes(int64_t rows, int64_t cols);

/*
 * out[c] = sum over r of src[r * ld + c], fp32 accumulation in a fixed order
 * (deterministic), written as `out_dtype`. `workspace` must hold
 * mb_column_sums_workspace_bytes(rows, cols) bytes (4-byte aligned).
 * Replaces: the bias gradient of src/myelin/triton/lif.py:1231-1258 (and
 *   grad_bias = grad.sum(...) of src/myelin/autograd.py:536-556).
 */
int mb_column_sums(int dtype, const void* src, int64_t rows, int64_t cols, int64_t ld,
                   int out_dtype, void* out, void* workspace, int64_t workspace_bytes,
                   void* stream);

/*
 * Pack spikes[rows, n] (any dtype; nonzero = spike, -0.0 counts as zero) into
 * int32 words[rows, ceil(n/32)], LSB-first, zero padding bits.
 * Replaces: packing.pack_spikes (src/myelin/packing.py:45-71) and
 *   triton/packing.py:20-41,100-131.
 */
int mb_pack_spikes(int dtype, const void* spikes, int32_t* words, int64_t rows, int64_t n,
                   void* stream);

/*
 * Unpack words[rows, ceil(n/32)] into out[rows, n] of `dtype` (0/1 values).
 * Replaces: packing.unpack_spikes (packing.py:74-81), triton/packing.py:44-66,134-175.
 */
int mb_unpack_spikes(const int32_t* words, int dtype, void* out, int64_t rows, int64_t n,
                     void* stream);

/*
 * Per-row spike counts (reduction over the last dimension, padding bits
 * ignored): counts[rows] int64.
 * Replaces: packing._packed_spike_row_counts (packing.py:165-206),
 *   triton/packing.py:69-91,178-225.
 */
int mb_count_rows(const int32_t* words, int64_t rows, int64_t n, int64_t* counts,
                  void* stream);

/*
 * Workspace (bytes, device memory) that mb_count_columns needs for
 * words[rows, ceil(n/32)]: one int32 partial count per (row slice, neuron).
 */
int64_t mb_count_columns_workspace_bytes(int64_t rows, int64_t n);

/*
 * Per-neuron spike counts summed over all leading rows (the dim=(0..nd-2)
 * reduction): counts[n]. Writes int64 to counts64 and/or int32 to counts32
 * (either may be NULL). Deterministic (integer arithmetic, fixed slice order).
 * `workspace` must hold mb_count_columns_workspace_bytes(rows, n) bytes,
 * 4-byte aligned; it is overwritten.
 * Replaces: packing._packed_spike_counts_over_leading_dims (packing.py:209-216).
 */
int mb_count_columns(const int32_t* words, int64_t rows, int64_t n, int64_t* counts64,
                     int32_t* counts32, void* workspace, int64_t workspace_bytes,
                     void* stream);

/* Workspace (bytes, device memory) that mb_pack_count_spikes needs (used by
 * the pack-then-count path; the one-pass path adds each row slice's counts
 * straight into the totals with integer atomics). */
int64_t mb_pack_count_workspace_bytes(int64_t rows, int64_t n);

/*
 * Pack spikes[rows, n] into words (as mb_pack_spikes) and count spikes per
 * neuron over all rows (as mb_count_columns on the words) in one call. For
 * aligned 1-byte spikes (bool / uint8 / int8) with n % 32 == 0 this is one
 * pass over the spikes; other inputs run the pack and the count kernels in
 * sequence. Same results either way (integer sums: exact in any order).
 * `workspace` must hold mb_pack_count_workspace_bytes(rows, n) bytes.
 * Replaces: the pair packing.pack_spikes (src/myelin/packing.py:45-71) +
 *   _packed_spike_counts_over_leading_dims (packing.py:209-216) that one
 *   step of a packed-spike all-gather / count all-reduce runs
 *   (distributed.py:63-109).
 */
int mb_pack_count_spikes(int dtype, const void* spikes, int32_t* words, int64_t rows, int64_t n,
                         int64_t* counts64, int32_t* counts32, void* workspace,
                         int64_t workspace_bytes, void* stream);

/*
 * Pack + per-neuron count (as mb_pack_count_spikes) whose packed words are
 * stored to `words` (this rank's [rows, ceil(n/32)] slot of its own gather
 * buffer) and to `num_peers` (0..7) more places: `peers` is a host array of
 * device pointers, each the start of this rank's slot in another rank's
 * gather buffer (mapped with mb_ipc_open; the stores go over NVLink). The
 * kernel reads the spikes once and writes every destination as it goes, so
 * the all-gather's transfers overlap the packing. It does not wait for
 * peers: the caller orders later reads of the gather buffers after every
 * rank's call (the count all-reduce that follows does that). Fused for
 * aligned 1-byte spikes with n % 32 == 0; other inputs pack into `words` and
 * a second kernel stores it into every peer slot.
 * Replaces: packing.pack_spikes + distributed.packed_spike_all_gather
 *   (src/myelin/distributed.py:63-80) + the local count of
 *   packed_spike_count_all_reduce (distributed.py:83-98).
 */
int mb_pack_count_scatter(int dtype, const void* spikes, int32_t* words, int64_t rows,
                          int64_t n, void* const* peers, int num_peers, int64_t* counts64,
                          int32_t* counts32, void* workspace, int64_t workspace_bytes,
                          void* stream);

/*
 * Gather buffers shared between the processes of a job through CUDA IPC (no
 * reference counterpart: the reference's all-gather is NCCL's). mb_ipc_alloc
 * allocates `bytes` on the current device and writes its IPC handle
 * (mb_ipc_handle_bytes() bytes) to `handle`; another process maps it with
 * mb_ipc_open and unmaps it with mb_ipc_close; the owner frees it with
 * mb_ipc_free.
 */
int mb_ipc_handle_bytes(void);
int mb_ipc_alloc(int64_t bytes, void** ptr, void* handle);
int mb_ipc_open(const void* handle, void** ptr);
int mb_ipc_close(void* ptr);
int mb_ipc_free(void* ptr);

/* Largest scratch (bytes) mb_count_columns_noalloc can use: 4 MiB. */
#define MB_COUNT_COLUMNS_NOALLOC_MAX_BYTES (4 << 20)

/*
 * mb_count_columns for callers that cannot allocate device memory when they
 * count: for example code running under a host runtime that owns all device
 * memory through its own fixed arena, or a latency-critical loop in which an
 * allocation call would block on the device. The per-slice partial sums live
 * in a fixed device array inside the library (MB_COUNT_COLUMNS_NOALLOC_MAX_BYTES,
 * held on every GPU that loads the library until the process exits), so the
 * caller passes only the words and the outputs. Same results as
 * mb_count_columns. Shapes whose scratch (mb_count_columns_workspace_bytes)
 * exceeds the limit are rejected with an error; the call allocates nothing.
 * The first call on each device looks up the array's device address (a
 * one-time set-up); make that first call before any stream capture. All calls
 * share the array: calls whose kernels overlap on the GPU race and give wrong
 * counts, so keep them ordered on one stream.
 * No counterpart in the reference.
 */
int mb_count_columns_noalloc(const int32_t* words, int64_t rows, int64_t n, int64_t* counts64,
                             int32_t* counts32, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MYELIN_B200_H */
