/*
 * libdotl: the C ABI of the B200 (sm_100a) single-transformer-layer forward.
 *
 * Every entry point takes plain device pointers, sizes and strides, and a
 * cudaStream_t passed as `void* stream`. No compute entry point allocates
 * device memory or synchronises (the peer-memory setup calls below do): outputs and temporaries are the caller's, and work
 * is enqueued on `stream` (so the calls can be captured in a CUDA graph).
 *
 * Return value: 0 on success; a nonzero DOTL_E* code otherwise, with a
 * message for the calling thread in dotl_last_error(). A rejected call
 * enqueues nothing.
 *
 * Each declaration names the reference entry point it replaces
 * (jazwinn/Distraction-OptimizedTransformerLayer, pybind module
 * `transformer_kernels`, csrc/fused_attention.cu:118-376). The reference binds
 * torch tensors through pybind; this ABI takes their data pointers, so any FFI
 * (ctypes, cffi, cgo, JNI) can bind it. The Python binding that rebuilds the
 * reference's tensor-level functions on top of it is
 * distraction-optimizedtransformerlayer_b200/dotl_ops.py.
 */
#ifndef DOTL_H_
#define DOTL_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DOTL_ABI_VERSION 2

/* status codes */
#define DOTL_OK 0
#define DOTL_EINVAL 1      /* an argument is out of the supported range */
#define DOTL_EUNSUPPORTED 2 /* a valid request no kernel here covers */
#define DOTL_ECUDA 3       /* the CUDA runtime/driver reported an error */

/* element types */
#define DOTL_F32 0
#define DOTL_F16 1
/*
 * An fp16 pair: a [rows, cols] tensor v stored as two fp16 planes of
 * [rows, ld] each, back to back: hi = fp16(v) (round to nearest even) in plane
 * 0 and lo = fp16(v - hi) in plane 1, starting rows * ld elements after plane
 * 0. hi + lo carries v to about 22 bits. GEMMs given DOTL_F16X2 operands run
 * three passes into one fp32 accumulator, a_hi w_hi + a_lo w_hi + a_hi w_lo
 * (the three-product mode: 3x the tensor work, for layer stacks whose fp16
 * operand error would otherwise exceed the harness's bound).
 */
#define DOTL_F16X2 2

/* dotl_linear residual modes */
#define DOTL_RESID_NONE 0        /* out = act(a w^T + bias) */
#define DOTL_RESID_ADD 1         /* out = resid + (a w^T + bias) */
#define DOTL_RESID_ADD_MASKSUB 2 /* out = resid + (valid ? a w^T + bias : 0) */
#define DOTL_RESID_ADD_MASKALL 3 /* out = valid ? resid + a w^T + bias : 0 */
#define DOTL_MASK_ROWS 4         /* out = valid ? act(a w^T + bias) : 0 (no residual) */

/* dotl_attention mask kinds */
#define DOTL_MASK_NONE 0
#define DOTL_MASK_KEY 1  /* per-key bool: mask[b*ms[0] + key*ms[3]], 1 = may attend */
#define DOTL_MASK_FULL 2 /* bool [B,H,S,S] via strides ms[0..3], 1 = may attend */

int dotl_abi_version(void);

/* Message for the last failed call on this thread ("" if none). */
const char* dotl_last_error(void);

/* Number of SMs of the current device (for sizing persistent grids). */
int dotl_num_sms(int* out);

/*
 * Sticky device-side error word. Kernels that give up a bounded wait (two
 * seconds on an mbarrier) set a bit here instead of hanging. Reading it
 * synchronises the current device. clear != 0 resets it.
 */
int dotl_device_error(int clear, unsigned int* word);

/* Copies n floats. Replaces smoke_test_identity (fused_attention.cu:97-116). */
int dotl_identity_f32(const float* in, float* out, int64_t n, void* stream);

/* fp32 -> fp16 (round to nearest even) and back, elementwise. */
int dotl_cast_f32_f16(const float* in, void* out_f16, int64_t n, void* stream);
int dotl_cast_f16_f32(const void* in_f16, float* out, int64_t n, void* stream);

/*
 * Residual add + LayerNorm over the last dimension of a [rows, D] fp32 tensor.
 * Replaces fused_add_layernorm (sub != NULL) and fused_layernorm (sub == NULL)
 * (add_layernorm.cuh:663-692; pybind fused_attention.cu:149-164).
 *   x_new  = x + sub                 written when sub and x_new are non-NULL
 *   normed = LN(x_new) * weight + bias, stored as fp32 or fp16 (normed_dtype)
 *   row_valid (optional, [rows] uint8): rows with 0 get normed = 0
 * normed_dtype DOTL_F32, DOTL_F16 or DOTL_F16X2 (normed then holds 2 * rows
 * rows: the hi plane, then the lo plane). All row pointers must be 16-byte
 * aligned for the vectorised path; other alignments take a scalar path.
 * D <= 2048.
 */
int dotl_layernorm(const float* x, const float* sub, const float* weight, const float* bias,
                   float* x_new, void* normed, int normed_dtype, const uint8_t* row_valid,
                   int64_t rows, int64_t D, float eps, void* stream);

/*
 * out[M,N] = epilogue(a[M,K] w[N,K]^T + bias[N]) with fp16 a and w, fp32
 * accumulation on tcgen05 tensor cores. Replaces linear_bias and linear_gelu
 * (linear_gelu.cuh:598-756; pybind fused_attention.cu:129-148).
 *   act: 0 none, 1 exact erf GELU (applied before any residual)
 *   resid_mode: DOTL_RESID_*; resid is fp32 [M, ldr]; row_valid [M] uint8
 *   out_dtype: DOTL_F32, DOTL_F16 or DOTL_F16X2 (fp16 pair, out holding 2 * M
 *              rows of ldo), leading dimension ldo
 *   operands: DOTL_F16 (a, w fp16), or DOTL_F16X2 (a is an fp16 pair of 2 * M
 *             rows of lda and w one of 2 * N rows of ldw; the three-product mode)
 * Requirements: K % 8 == 0, lda % 8 == 0, ldw % 8 == 0, a/w 16-byte aligned
 * (TMA), N % 8 == 0. tile_n: 0 = auto, else 64, 128, 160, 192, 224 or 256
 * (the widths between the powers of two fill a last wave of tiles that 128 or
 * 256 would leave partly idle; every width gives the same bits), or -128 for two
 * CTAs per 128-wide tile that split K and add their partial sums (auto picks it
 * for long K when the tiles cannot fill the SMs; the add is one fp32 sum, so
 * results are the same on every run), or -256 for 256 x 256 tiles on CTA pairs
 * (cta_group::2 MMAs with M = 256; the same bits as tile_n 256; auto picks it
 * for fp32 residual outputs with N >= 2048, K >= 2048 and at least four pair
 * tiles per pair of SMs).
 */
int dotl_linear(const void* a, int64_t M, int64_t K, int64_t lda, const void* w, int64_t N,
                int64_t ldw, const float* bias, int act, const float* resid, int64_t ldr,
                const uint8_t* row_valid, int resid_mode, void* out, int out_dtype, int64_t ldo,
                int tile_n, int operands, void* stream);

/*
 * dotl_linear with a residual + LayerNorm epilogue, in one kernel. Replaces the
 * pairs linear_bias -> fused_add_layernorm / fused_layernorm of the layer
 * (linear_gelu.cuh:598-756 then add_layernorm.cuh:663-692):
 *   x_new  = resid_mode epilogue(a w^T + bias)   fp32; stored to out unless out == NULL
 *   normed = LN(x_new) * ln_weight + ln_bias      over all N columns, eps as given
 *   normed_row_valid (optional, [M] uint8): rows with 0 get normed = 0
 * resid_mode: NONE, ADD, ADD_MASKSUB or ADD_MASKALL (as dotl_linear; row_valid
 * for the masked ones). normed_dtype DOTL_F32, DOTL_F16 or DOTL_F16X2 (2 * M rows
 * of ldn), leading dimension ldn; operands as dotl_linear.
 * The row is shared by a cluster of N / tile_n CTAs, so N must be 64, 128 or
 * 256 times a cluster size of at most 8 (tile_n 0 = auto). Other requirements
 * as dotl_linear; ln_weight and ln_bias 16-byte aligned.
 */
int dotl_linear_ln(const void* a, int64_t M, int64_t K, int64_t lda, const void* w, int64_t N,
                   int64_t ldw, const float* bias, const float* resid, int64_t ldr,
                   const uint8_t* row_valid, int resid_mode, float* out, int64_t ldo,
                   const float* ln_weight, const float* ln_bias, float eps, void* normed,
                   int normed_dtype, int64_t ldn, const uint8_t* normed_row_valid, int tile_n,
                   int operands, void* stream);

/*
 * The layer's whole MLP in one kernel, the [M, F] hidden kept on chip.
 * Replaces linear_gelu -> linear_bias -> fused_add_layernorm (linear_gelu.cuh:
 * 598-756, add_layernorm.cuh:663-692; the sequence of optimized/layers.py:
 * 241-261) and supersedes fused_ffn_block (ffn_block.cuh:270-311, which covers
 * only d = F <= 64):
 *   h      = GELU_erf(a w1^T + b1)              a fp16 [M, D]; h rounded to fp16, never stored
 *   x_new  = resid_mode epilogue(h w2^T + b2)   as dotl_linear; stored to x_out unless NULL
 *   normed = LN(x_new) * ln_weight + ln_bias     0 where normed_row_valid is 0
 * w1 fp16 [F, D], w2 fp16 [D, F] (nn.Linear layouts). D (d_model) 128 or 256;
 * F a multiple of 128. resid_mode NONE, ADD, ADD_MASKSUB or ADD_MASKALL.
 * Leading dimensions multiples of 8 (4 for the fp32 ones), pointers 16-byte aligned.
 */
int dotl_ffn(const void* a, int64_t M, int64_t D, int64_t lda, const void* w1, int64_t F, int64_t ldw1,
             const float* b1, const void* w2, int64_t ldw2, const float* b2, const float* resid, int64_t ldr,
             const uint8_t* row_valid, int resid_mode, float* x_out, int64_t ldx, const float* ln_weight,
             const float* ln_bias, float eps, void* normed, int normed_dtype, int64_t ldn,
             const uint8_t* normed_row_valid, void* stream);

/*
 * Flash attention forward, fp16 q/k/v, fp32 softmax, fp16 output.
 * Replaces fused_attention_forward (attention_dispatch.cuh:332-519).
 *   q/k/v: [B,H,S,head_dim] addressed by {batch, head, seq} element strides
 *          (head_dim stride 1), 16-byte aligned, strides multiples of 8.
 *   mask_kind: DOTL_MASK_*; mask strides ms[4] in elements (b, h, query, key).
 *   causal: key j may be attended by query i only if j <= i (combinable).
 *   out: fp16, layout 0 = [B,H,S,head_dim], 1 = [B,S,H*head_dim]; out_dtype
 *        DOTL_F16, or DOTL_F16X2 (the lo plane follows, B*H*S*head_dim later).
 * Fully masked query rows are written as 0. head_dim 32, 64 or 128 run on the
 * tcgen05 kernel; other multiples of 8 up to 256 on a CUDA-core flash kernel
 * (the reference's scalar/wmma shapes, e.g. head_dim 8 and 256).
 *   workspace: NULL, or at least dotl_attention_workspace_bytes(...) bytes of
 *   16-byte-aligned device memory. Given one, shapes with too few (batch,
 *   head, 128-row query tile) items to fill the SMs and long key ranges run
 *   split-KV: each tile's keys in runs on separate CTAs, then a combine
 *   kernel folds the runs (the reference's split-KV path and its combine,
 *   attention_wmma.cuh:662-759, 1783-1826). Same results either way to
 *   fp32 rounding; repeat calls give the same bits.
 */
int dotl_attention(const void* q, const void* k, const void* v, int B, int H, int S, int head_dim,
                   const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                   const uint8_t* mask, int mask_kind, const int64_t* mask_strides, int causal,
                   float scale, void* out, int out_layout, int out_dtype, void* workspace,
                   int64_t workspace_bytes, void* stream);

/*
 * Workspace dotl_attention would use for split-KV on this shape on the current
 * device (0: it would not split). Replaces the caching-allocator workspace of
 * the reference's split path (attention_wmma.cuh:1925-1937).
 */
int dotl_attention_workspace_bytes(int B, int H, int S, int head_dim, int causal, int64_t* bytes);

/*
 * dotl_attention without a caller workspace, for callers that cannot allocate
 * device memory themselves: a host binding with no CUDA allocator of its own
 * to call, or code running where growing device memory is not allowed. It
 * allocates nothing. The split-KV scratch is one static device array of
 * DOTL_ATTENTION_STATIC_SCRATCH_BYTES per device, held by every GPU that loads
 * the library until the process exits. Shapes whose split plan needs more
 * (dotl_attention_workspace_bytes above the limit) are rejected with
 * DOTL_EUNSUPPORTED; shapes that need none run the one-pass kernel. Every call
 * on a device uses the same array: calls whose kernels may overlap on the GPU
 * (other streams, other threads) race on it, so serialise them, e.g. on one
 * stream. Each call writes every scratch word it reads, so nothing needs
 * clearing between calls. The first call on a device looks up the array's
 * device address (with that device current); make it before any stream
 * capture. Otherwise the same arguments and results as dotl_attention.
 * No counterpart in the reference.
 */
#define DOTL_ATTENTION_STATIC_SCRATCH_BYTES (16 << 20)
int dotl_attention_static_scratch(const void* q, const void* k, const void* v, int B, int H, int S, int head_dim,
                                  const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                                  const uint8_t* mask, int mask_kind, const int64_t* mask_strides, int causal,
                                  float scale, void* out, int out_layout, int out_dtype, void* stream);

/*
 * Peer memory for the tensor-parallel layer (one process per GPU). These are
 * setup calls, made once per peer group, and the only entry points that
 * allocate or map device memory:
 *   dotl_peer_alloc    cudaMalloc'd, zeroed buffer whose IPC handle peers can open
 *   dotl_ipc_handle    its handle (DOTL_IPC_HANDLE_BYTES opaque bytes) for the peers
 *   dotl_ipc_open      maps a peer's buffer into this process (peer access enabled)
 *   dotl_ipc_close / dotl_peer_free undo them (close peers' mappings first)
 *   dotl_peer_blocks   the grid dotl_allreduce_ln may use on this device (every CTA
 *                      resident at once); all ranks must pass the same value
 *   dotl_peer_signal_bytes  size of one rank's signal area for that grid
 * No reference counterpart: the reference runs on one GPU.
 */
#define DOTL_IPC_HANDLE_BYTES 64
int dotl_peer_alloc(int64_t bytes, void** ptr);
int dotl_peer_free(void* ptr);
int dotl_ipc_handle(const void* ptr, void* handle);
int dotl_ipc_open(const void* handle, void** ptr);
int dotl_ipc_close(void* ptr);
int dotl_peer_blocks(int* blocks);
int dotl_peer_signal_bytes(int blocks, int64_t* bytes);

/*
 * dotl_linear (fp32 out, optional bias, no residual or activation) whose
 * output tiles go to the rank that owns their rows, for the row-parallel GEMMs
 * of the tensor-parallel layer: row block m goes to rank (128 m) / rows_per_rank,
 * at row 128 m - rank * rows_per_rank of outs[rank]. outs[i] is this rank's
 * receive slot on rank i (peer-mapped with dotl_ipc_open; outs[own rank] its own
 * memory). The stores are TMA bulk stores over NVLink, issued from the GEMM's
 * epilogue while its tensor cores run the next tile: the reduce-scatter of
 * all_reduce(part) (optimized/layers.py:241-243, 258-261 on one GPU) moves
 * inside the GEMM, and dotl_allreduce_ln (parts_local = 1) finishes the
 * reduction from local memory. M = world * rows_per_rank, rows_per_rank % 128
 * == 0, world <= 8; other requirements as dotl_linear. The receive slots must
 * not be read until every rank's GEMM is complete (dotl_allreduce_ln's start
 * handshake ensures it).
 */
int dotl_linear_peer(const void* a, int64_t M, int64_t K, int64_t lda, const void* w, int64_t N, int64_t ldw,
                     const float* bias, int world, void* const* outs, int64_t rows_per_rank, int64_t ldo,
                     void* stream);

/*
 * Sum over the ranks of fp32 partial sums + bias + residual + LayerNorm, in one
 * kernel over peer memory. Replaces all_reduce(part) followed by
 * fused_add_layernorm (add_layernorm.cuh:663-672) after each row-parallel GEMM
 * of the tensor-parallel layer (the single-GPU pairs are optimized/layers.py:
 * 241-243 and 258-261):
 *   sum    = parts[0] + ... + parts[world-1] (+ bias)   in rank order: same bits on every rank
 *   x_new  = x + (sum_row_valid ? sum : 0)              fp32; not stored where x_new[i] is NULL
 *   normed = LN(x_new) * ln_weight + ln_bias            0 on rows normed_row_valid marks 0
 * parts / signals / x_new / normed are host arrays of `world` device pointers,
 * entry i being rank i's buffer as this process sees it (its own, or a peer's
 * mapped by dotl_ipc_open); signal areas are zeroed dotl_peer_alloc memory of
 * dotl_peer_signal_bytes(blocks). push = 0: this rank computes every row and
 * writes only x_new[rank] / normed[rank]. push = 1: rank r computes rows
 * [r*ceil(rows/world), ...) and writes them into every rank's outputs (which
 * must then be peer-mapped too). parts_local = 1 (push only): parts[i] is instead
 * this rank's own slot holding rank i's partial sums of this rank's rows (row
 * r0 of the slice at offset 0), as dotl_linear_peer leaves them, so only the
 * results cross NVLink. Every rank must make the same calls with the
 * same rows, D, push and blocks, in the same order. blocks must be the value
 * the signal areas were sized for (signal_bytes = dotl_peer_signal_bytes(blocks),
 * checked: the layout depends on it), the same on every call and every rank. A
 * wait for a peer longer than timeout_ms sets bit 4 of the device error word,
 * stores that bit into *status when status is not NULL (any device-visible word:
 * host-mapped pinned memory lets the host see it without a device sync), and
 * ends the call's work; the group's counters then disagree and it must be
 * rebuilt. D % 4 == 0, D <= 2048, world <= 8, all pointers 16-byte aligned.
 */
int dotl_allreduce_ln(int world, int rank, const float* const* parts, void* const* signals, float* const* x_new,
                      void* const* normed, int normed_dtype, int push, int parts_local, const float* x, const float* bias,
                      const uint8_t* sum_row_valid, const float* ln_weight, const float* ln_bias, float eps,
                      const uint8_t* normed_row_valid, int64_t rows, int64_t D, int blocks, int64_t signal_bytes,
                      unsigned int* status, int timeout_ms, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DOTL_H_ */
