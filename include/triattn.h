/*
 * triattn.h -- C ABI of the B200 (sm_100a) pairformer triangle-attention library (libtriattn.so).
 *
 * One triangle-attention layer (starting node or ending node, forward only) of Boltz-2's
 * pairformer: z[B,N,N,128] fp32, pair mask [B,N,N], 4 heads x 32 head dim, parameters under the
 * reference's names (layer_norm.{weight,bias}, linear.weight [4,128], mha.linear_{q,k,v,g,o}.weight).
 *
 * Conventions
 *   - Every pointer argument is a DEVICE pointer unless stated otherwise; the caller allocates every
 *     output, the packed weights and the workspace.  The library never allocates or frees memory
 *     except in triattn_peer_alloc / triattn_peer_free (buffers shared between GPUs).
 *   - `stream` is a cudaStream_t passed as void* (NULL = the legacy default stream).  Calls are
 *     asynchronous: they validate arguments on the host, enqueue kernels and return.
 *   - Tensors are dense and row-major ("contiguous"): z/out [B][N][N][128] fp32, mask [B][N][N] fp32.
 *   - Return value: TRIATTN_OK or an error code below.  No call traps or asserts on the device;
 *     kernels record device-side failures (a bounded wait that ran out) in a status word that
 *     triattn_device_status() reads.
 *   - dtype selects the arithmetic of the layer: TRIATTN_F32 = fp32 everywhere (SIMT, the
 *     reference's fp32 path, max-rel <= 1e-5); TRIATTN_F16 / TRIATTN_BF16 = 16-bit operands on the
 *     tcgen05 tensor cores with fp32 accumulation, fp32 softmax statistics and an fp32 residual.
 *
 * Reference interfaces replaced (paths inside jackryan225/boltz-mlx):
 *   triattn_forward      <- TriangleAttention.__call__        boltz_mlx/layers/triangular_attention/attention.py:27-93
 *                           (+ the residual add of PairformerLayer, boltz_mlx/layers/pairformer.py:86-87)
 *   triattn_mask_prep    <- nax_tri_inputs mask bias            boltz_mlx/kernels_nax.py:477-503 / attention.py:85
 *   triattn_ln_proj      <- layer_norm + fused projection       boltz_mlx/kernels.py:482-507, attention.py:47-53,69,
 *                           (pair_proj16 + tri-bias GEMM)       boltz_mlx/kernels_nax3.py:1625-1634, attention.py:145-149
 *   triattn_core         <- tri_attention_fused / tri_attention_nax  boltz_mlx/kernels.py:902-945,
 *                                                                     boltz_mlx/kernels_nax.py:506-558
 *   triattn_out_proj     <- linear_o / lin16 / linear_addln      attention.py:89, boltz_mlx/kernels.py:1287-1370,
 *                                                                 boltz_mlx/kernels_nax3.py:320-354
 *   triattn_pack_weights <- w16 fused fp16 weight cache          boltz_mlx/kernels.py:1349-1357
 */
#ifndef TRIATTN_H
#define TRIATTN_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TRIATTN_API __attribute__((visibility("default")))
#else
#define TRIATTN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------------------------- */
#define TRIATTN_OK 0
#define TRIATTN_EINVAL 1       /* null pointer, bad size, bad alignment, bad row range          */
#define TRIATTN_EUNSUPPORTED 2 /* dtype / configuration not supported by this build             */
#define TRIATTN_ECUDA 3        /* a CUDA runtime call or launch failed (triattn_last_error_string) */
#define TRIATTN_EDEVICE 4      /* a kernel recorded a device-side failure (bounded wait ran out) */
#define TRIATTN_ENOSPACE 5     /* workspace or packed-weight buffer too small                    */

/* ---- dtypes ------------------------------------------------------------------------------- */
#define TRIATTN_F32 0
#define TRIATTN_F16 1
#define TRIATTN_BF16 2

/* Fixed layer geometry of Boltz-2's triangle attention (attention.py:15, pairformer.py:51-52). */
#define TRIATTN_C_IN 128
#define TRIATTN_HEADS 4
#define TRIATTN_C_HEAD 32

/* Library version string (static storage). */
TRIATTN_API const char* triattn_version(void);

/* Human-readable text of the last host-side error on the calling thread (static storage). */
TRIATTN_API const char* triattn_last_error_string(void);

/* Read the device status word of the current device (0 = ok; 101 a bulk copy, 102 an MMA, 103 a
 * barrier wait ran out; 105 a shared-memory base was not aligned as a
 * swizzled operand needs; 106 a cross-GPU barrier missed a peer); clear it when `clear` != 0.
 * Synchronises the device.  Returns TRIATTN_OK and writes the word to *status. */
TRIATTN_API int triattn_device_status(int* status, int clear);

/* ---- weights ------------------------------------------------------------------------------ */
/* Bytes of the packed-weight buffer for `dtype`. */
TRIATTN_API size_t triattn_packed_weights_bytes(int dtype);

/* Pack one module's parameters (all DEVICE fp32, reference [out, in] Linear layout):
 *   ln_w, ln_b [128]; w_q, w_k, w_v, w_g [128,128]; g_bias [128] or NULL (the reference has none);
 *   w_b [4,128] (the module's `linear`, tri-bias projection); w_o [128,128].
 * Writes fp32 copies plus, for 16-bit dtypes, the tensor-core operand images of W_qkvg [512,128]
 * and W_o [128,128].  Done once per module; the result is reused by every call. */
TRIATTN_API int triattn_pack_weights(const float* ln_w, const float* ln_b, const float* w_q, const float* w_k,
                         const float* w_v, const float* w_g, const float* g_bias, const float* w_b,
                         const float* w_o, int dtype, void* packed, size_t packed_bytes, void* stream);

/* ---- workspace ---------------------------------------------------------------------------- */
/* Bytes of workspace for attention rows [row_begin, row_end) of a B x N layer (rows = row_end -
 * row_begin; the tri-bias region always covers all N rows).  Needs 256-byte alignment. */
TRIATTN_API size_t triattn_workspace_bytes(int B, int N, int rows, int dtype);

/* ---- one layer ---------------------------------------------------------------------------- */
/* out = y (add_residual = 0) or z + y (add_residual = 1), y = TriangleAttention(z, mask).
 * starting = 1: starting node; 0: ending node (attention over the transposed pair layout, read
 * and written in place -- z^T is never materialised).  mask may be NULL (all ones).  out may
 * alias z when add_residual = 1 (in-place residual stream).  inf: the reference's 1e9. */
TRIATTN_API int triattn_forward(const float* z, const float* mask, const void* packed, int B, int N, int starting,
                    float inf, int dtype, int add_residual, float* out, void* workspace, size_t workspace_bytes,
                    void* stream);

/* Row-chunked form of triattn_forward for large N (bounded memory) <- the reference's chunked layer
 * (attention.py:55-68: the tri bias from ALL rows, then the attention core over row chunks): pass 1
 * runs the LayerNorm + projection of every chunk for its tri-bias rows, pass 2 runs mask bias,
 * LayerNorm + projection, core and output projection chunk by chunk.  The workspace covers
 * chunk_rows rows only: triattn_workspace_bytes(B, N, chunk_rows, dtype) (the tri-bias region, which
 * always spans all N rows, plus chunk_rows rows of per-row regions).  chunk_rows >= N is one chunk;
 * on the 16-bit path a smaller chunk_rows must be a multiple of 128.  Results equal
 * triattn_forward's bit for bit (identical per-row arithmetic); out may alias z (add_residual = 1).
 * All offsets are 64-bit: N up to 16384 (z alone is 137 GB there). */
TRIATTN_API int triattn_forward_chunked(const float* z, const float* mask, const void* packed, int B, int N,
                                        int starting, float inf, int dtype, int add_residual, float* out,
                                        int chunk_rows, void* workspace, size_t workspace_bytes, void* stream);

/* ---- stages (row-range granularity: the reference's row chunking, attention.py:55-68) ------
 * All stages address attention rows a in [row_begin, row_end) of the full-size z / mask / out. */

/* Mask bias of the attention rows: inf * (mask - 1) per (row, key), keys padded to a tile. */
TRIATTN_API int triattn_mask_prep(const float* mask, int B, int N, int starting, float inf, int row_begin, int row_end,
                      int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* LayerNorm + q|k|v|g projection of rows [row_begin,row_end) and their tri-bias rows. */
TRIATTN_API int triattn_ln_proj(const float* z, const void* packed, int B, int N, int starting, int row_begin, int row_end,
                    int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* Flash attention core with tri bias, mask bias, online softmax and sigmoid gate; needs the
 * tri-bias rows of ALL N rows in the workspace. */
TRIATTN_API int triattn_core(int B, int N, int row_begin, int row_end, int dtype, void* workspace, size_t workspace_bytes,
                 void* stream);

/* Fused-neighbour form of triattn_forward <- TriangleAttention._f16 / f16_addln
 *   (boltz_mlx/layers/triangular_attention/attention.py:95-103,170-190; kernels_nax3.linear_addln
 *   kernels_nax3.py:69-198; pair block kernels.py:1526-1547), 16-bit dtypes only:
 *   xn       : NULL -> LayerNorm of z as in triattn_forward; else this layer's LayerNorm output
 *              [B][N][N][128] in the layer's 16-bit type, laid out in the layer's attention orientation
 *              (for the ending node already transposed, as the reference passes it); z is then read
 *              only for the residual.
 *   out_attn_layout : 0 -> out in z's orientation; 1 -> in the layer's attention orientation (the
 *              reference's keep_t for the ending node).
 *   ln_out   : NULL, or [B][N][N][128] 16-bit <- LayerNorm(ln_next_w, ln_next_b, eps 1e-5) of every
 *              output row (the next module's input), in z's orientation (ln_out_swapped = 0) or with
 *              the two N axes swapped (1; the reference's trans_out). */
TRIATTN_API int triattn_forward_fused(const float* z, const void* xn, const float* mask, const void* packed, int B,
                                      int N, int starting, float inf, int dtype, int add_residual, float* out,
                                      int out_attn_layout, const float* ln_next_w, const float* ln_next_b,
                                      void* ln_out, int ln_out_swapped, void* workspace, size_t workspace_bytes,
                                      void* stream);
/* triattn_forward_fused with the pair block's tri-bias hand-over <- the reference's tb / w_tb arguments
 *   of f16_addln (attention.py:170-190, consumed by _f16_core at :128-147; kernels.py:1537-1539) and the
 *   PAIRTB LayerNorm epilogue (_LN_EPI_TB, kernels_nax3.py:104-143):
 *   tb        : NULL, or (with xn) this layer's tri bias as computed by the producer of xn, fp16
 *               [B][4][N][N] in natural units, laid out like xn (the layer's attention orientation);
 *               the projection then takes it instead of its own LN . w_b dot.
 *   tb_next_w : fp32 [4][128], the next triangle attention's tri-bias weight; with ln_out and tb_next,
 *   tb_next   : fp16 [B][4][N][N] <- sum_c ln_out[pair][c] * tb_next_w[h][c] over the ROUNDED 16-bit
 *               ln_out values, fp32 sums, one rounding; pairs in ln_out's order (ln_out_swapped included).
 * Every other argument as triattn_forward_fused, which is this call with tb = tb_next_w = tb_next = NULL. */
TRIATTN_API int triattn_forward_fused_tb(const float* z, const void* xn, const void* tb, const float* mask,
                                         const void* packed, int B, int N, int starting, float inf, int dtype,
                                         int add_residual, float* out, int out_attn_layout, const float* ln_next_w,
                                         const float* ln_next_b, void* ln_out, int ln_out_swapped,
                                         const float* tb_next_w, void* tb_next, void* workspace,
                                         size_t workspace_bytes, void* stream);

/* ---- strided-view stages (row-sharded / column-blocked pair tensors) ------------------------
 * The _v variants address an attention-oriented VIEW of a pair tensor instead of a dense [B][N][N]
 * one: element (b, a, c, ch) of the view lives at
 *     base + b*s_batch + (a - row_begin)*s_row + c*s_col + ch          (in elements)
 * for attention rows a in [row_begin, row_end) and columns c in [0, N).  For the pair tensors
 * s_row and s_col must be multiples of 4 (16-byte rows).  A rank that owns rows [r0, r1) of z
 * passes its local shard with s_row = N*128, s_col = 128; after an all-to-all it owns columns and
 * passes the received block with s_row = 128, s_col = rows_per_rank*128. */
TRIATTN_API int triattn_mask_prep_v(const float* mask, int64_t s_batch, int64_t s_row, int64_t s_col, int B, int N,
                                    float inf, int row_begin, int row_end, int dtype, void* workspace,
                                    size_t workspace_bytes, void* stream);
TRIATTN_API int triattn_ln_proj_v(const float* z, int64_t s_batch, int64_t s_row, int64_t s_col, const void* packed,
                                  int B, int N, int row_begin, int row_end, int dtype, void* workspace,
                                  size_t workspace_bytes, void* stream);
TRIATTN_API int triattn_out_proj_v(const float* z, int64_t zs_batch, int64_t zs_row, int64_t zs_col, float* out,
                                   int64_t os_batch, int64_t os_row, int64_t os_col, const void* packed, int B, int N,
                                   int row_begin, int row_end, int dtype, int add_residual, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* Column-blocked views (no reference counterpart: the layout of a row-sharded residual stream).
 * Column c of the view lives at (c / col_block)*s_col_block + (c % col_block)*s_col instead of
 * c*s_col (col_block = 0: plain view).  A rank owning rows [r0, r0 + R) keeps its rows of z as
 * [P][R][R][128] blocks (block p = columns of rank p): s_row = R*128, s_col = 128, col_block = R,
 * s_col_block = R*R*128.  Block p is then exactly what all_to_all_single sends to rank p, and what
 * comes back from the ending node lands in the same layout: the exchange needs no transposing copy. */
TRIATTN_API int triattn_ln_proj_vb(const float* z, int64_t s_batch, int64_t s_row, int64_t s_col, int col_block,
                                   int64_t s_col_block, const void* packed, int B, int N, int row_begin, int row_end,
                                   int dtype, void* workspace, size_t workspace_bytes, void* stream);
TRIATTN_API int triattn_out_proj_vb(const float* z, int64_t zs_batch, int64_t zs_row, int64_t zs_col,
                                    int z_col_block, int64_t zs_col_block, float* out, int64_t os_batch,
                                    int64_t os_row, int64_t os_col, int o_col_block, int64_t os_col_block,
                                    const void* packed, int B, int N, int row_begin, int row_end, int dtype,
                                    int add_residual, void* workspace, size_t workspace_bytes, void* stream);

/* ---- peer-store exchange (one process per GPU of a node) -------------------------------------
 * No reference counterpart: the reference runs on one device and bounds memory by row chunking
 * (attention.py:55-68).  A row-sharded layer hands its output blocks to the ranks that consume them
 * by storing them into those ranks' memory over NVLink from inside the output projection, instead of
 * an all-to-all after it.  Shared buffers come from triattn_peer_alloc (a zero-filled allocation of
 * their own, so an IPC handle maps exactly the buffer); the caller exchanges the 64-byte handles
 * (an all-gather on its process group) and opens every other rank's with triattn_ipc_open.  Close
 * the mappings on every rank before any owner frees its buffer. */
#define TRIATTN_IPC_HANDLE_BYTES 64
TRIATTN_API int triattn_peer_alloc(size_t bytes, void** dev_ptr);
TRIATTN_API int triattn_peer_free(void* dev_ptr);
TRIATTN_API int triattn_ipc_handle(void* dev_ptr, void* handle);
TRIATTN_API int triattn_ipc_open(const void* handle, void** dev_ptr);
TRIATTN_API int triattn_ipc_close(void* dev_ptr);

/* Output projection (+ residual) whose column blocks lie anywhere in this process's address space
 * (mapped peer buffers included): column c of the output view lives at
 *     out + o_block_table[c / o_col_block] + (c % o_col_block)*os_col       (in elements)
 * o_block_table is DEVICE memory, N / o_col_block int64 entries (element offsets from out; peer
 * mappings give offsets outside out's own allocation).  The z view is as in triattn_out_proj_vb.
 * Every store is made visible system-wide before the kernel ends; a triattn_peer_barrier after it on
 * the same stream publishes the blocks to their owners. */
TRIATTN_API int triattn_out_proj_vt(const float* z, int64_t zs_batch, int64_t zs_row, int64_t zs_col,
                                    int z_col_block, int64_t zs_col_block, float* out, int64_t os_batch,
                                    int64_t os_row, int64_t os_col, int o_col_block, const int64_t* o_block_table,
                                    const void* packed, int B, int N, int row_begin, int row_end, int dtype,
                                    int add_residual, void* workspace, size_t workspace_bytes, void* stream);

/* Copy bytes [offset, offset + bytes) of this rank's shared buffer to the same range of every other
 * rank's (buf_ptrs: DEVICE array of `world` uint64 buffer addresses as mapped here; offset and bytes
 * multiples of 16).  One launch, all peers' links at once; the row-sharded layer hands its tri-bias
 * rows to every rank this way.  Publish with triattn_peer_barrier. */
TRIATTN_API int triattn_peer_broadcast(const uint64_t* buf_ptrs, int rank, int world, size_t offset, size_t bytes,
                                       void* stream);

/* Cross-GPU barrier on `stream`.  flag_ptrs: DEVICE array of `world` uint64 addresses, entry t = rank
 * t's flag block (world 32-bit slots, zero-filled at start) as mapped in this process.  Every rank
 * calls it with the same epoch sequence (1, 2, 3, ...).  Bounded: a peer that does not arrive within
 * 2 s leaves device status 106 (triattn_device_status) and the kernel returns. */
TRIATTN_API int triattn_peer_barrier(const uint64_t* flag_ptrs, int rank, int world, uint32_t epoch, void* stream);

/* Output projection (+ residual) of rows [row_begin,row_end), written in z's orientation. */
TRIATTN_API int triattn_out_proj(const float* z, const void* packed, int B, int N, int starting, int row_begin, int row_end,
                     int dtype, int add_residual, float* out, void* workspace, size_t workspace_bytes,
                     void* stream);

/* ---- triangle multiplication (the pairformer's other O(N^3) pair op) -----------------------
 * TriangleMultiplicationOutgoing / Incoming <- boltz_mlx/layers/triangular_mult.py:10-178 (fp32 ops
 * path :23-49; parameters norm_in.{weight,bias}, p_in.weight [256,128], g_in.weight [256,128],
 * norm_out.{weight,bias}, p_out.weight [128,128], g_out.weight [128,128], no biases):
 *   xn = norm_in(z); a|b = p_in(xn) * sigmoid(g_in(xn)) * mask
 *   outgoing o[i,j,d] = sum_k a[i,k,d] b[j,k,d];  incoming o[i,j,d] = sum_k a[k,i,d] b[k,j,d]
 *   out = (z +) p_out(norm_out(o)) * sigmoid(g_out(xn))
 * dtype: TRIATTN_F32 (every step fp32) or a 16-bit type (operands 16-bit, fp32 accumulation, fp32 o).
 * mask may be NULL (ones); out may alias z with add_residual = 1.  B*N*N must stay below 2^31.
 * The contraction and the projections run as cuBLAS GEMMs on `stream`, with the workspace's last 32
 * MiB as cuBLAS scratch (the first call on a device creates its cuBLAS handle). */
TRIATTN_API size_t triattn_trimul_packed_bytes(int dtype);
TRIATTN_API int triattn_trimul_pack_weights(const float* in_w, const float* in_b, const float* p_in,
                                            const float* g_in, const float* out_w, const float* out_b,
                                            const float* p_out, const float* g_out, int dtype, void* packed,
                                            size_t packed_bytes, void* stream);
TRIATTN_API size_t triattn_trimul_workspace_bytes(int B, int N, int dtype);
TRIATTN_API int triattn_trimul_forward(const float* z, const float* mask, const void* packed, int B, int N,
                                       int outgoing, int dtype, int add_residual, float* out, void* workspace,
                                       size_t workspace_bytes, void* stream);
/* out = z + TriangleMultiplication(z) and ln_out = LN_next(out) in the layer's 16-bit type, from one
 * tail kernel <- the reference's f16_addln (triangular_mult.py:93-115, kernels_nax3.trimul_tail_addln):
 * the next module (a triangle attention, whose `xn` input this is) skips its LayerNorm.  16-bit
 * dtypes only; ln_out [B][N][N][128] in z's orientation; ln_next_w / ln_next_b fp32 [128]. */
TRIATTN_API int triattn_trimul_forward_addln(const float* z, const float* mask, const void* packed, int B, int N,
                                             int outgoing, int dtype, float* out, const float* ln_next_w,
                                             const float* ln_next_b, void* ln_out, void* workspace,
                                             size_t workspace_bytes, void* stream);
/* triattn_trimul_forward_addln that also writes the next triangle attention's tri bias <- the
 * reference's f16_addln(..., w_tb=...) of the tri-mult (kernels.py:1537, PAIRTB epilogue
 * kernels_nax3.py:104-143): tb_next fp16 [B][4][N][N] = sum_c ln_out[pair][c] * tb_next_w[h][c]
 * (tb_next_w fp32 [4][128]) over the rounded ln_out values, pairs in ln_out's (z's) order. */
TRIATTN_API int triattn_trimul_forward_addln_tb(const float* z, const float* mask, const void* packed, int B, int N,
                                                int outgoing, int dtype, float* out, const float* ln_next_w,
                                                const float* ln_next_b, void* ln_out, const float* tb_next_w,
                                                void* tb_next, void* workspace, size_t workspace_bytes,
                                                void* stream);

/* ---- allocation-free layer ----------------------------------------------------------------
 * No counterpart in the reference.  triattn_forward without a workspace argument, for callers that
 * cannot allocate device memory at run time (a plugin host that forbids cudaMalloc after start-up,
 * a process whose device memory is owned by another allocator, a fixed device footprint).  The
 * scratch is a 48 MiB array inside the library; a GPU holds it from the first call on that device
 * (CUDA's default lazy module loading reserves it then; eager loading at library load) until exit,
 * so make one small call per device at start-up, before handing memory to another allocator.  Calls
 * whose triattn_workspace_bytes(B, N, N, dtype) exceeds it (about N > 128 at B = 1) return
 * TRIATTN_ENOSPACE.  The first call on a device looks the array up (make it before any stream
 * capture); calls share the array, so calls that overlap on the GPU race.  Allocates nothing. */
TRIATTN_API int triattn_forward_noalloc(const float* z, const float* mask, const void* packed, int B, int N,
                                        int starting, float inf, int dtype, int add_residual, float* out,
                                        void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TRIATTN_H */
