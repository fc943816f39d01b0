/*
 * tinydeform.h -- C ABI of the B200 (sm_100a) ma_deform_attn library (libtinydeform / _tinydeform.so).
 *
 * The library computes value projection + multi-scale deformable attention for DETR-style decoders:
 *
 *   value[b, n, :]      = memory[b, n, :] @ value_weight^T + value_bias          ([B, N, H*D])
 *   out[b, q, h*D + d]  = sum over levels l, points p, bilinear corners k of
 *                         attention_weights[b,q,h,l,p] * bilinear_k * value[b, token_k, h*D + d]
 *
 * with bilinear sampling at (x*w_l - 0.5, y*h_l - 0.5) (grid_sample, align_corners=False) and zero padding:
 * corners outside a level's map contribute nothing.
 *
 * Conventions shared by every entry point:
 *   - All tensor pointers are DEVICE pointers on the current CUDA device, dense row-major (contiguous).
 *   - spatial_shapes is int64 [L, 2] (height, width); level_start_index is int64 [L]. Both stay on the device and
 *     are read by the kernels, so a call never synchronises with the host and can be captured in a CUDA graph.
 *   - dtype is one of TD_F32, TD_F16, TD_BF16, TD_F64; every float tensor of a call has that dtype. Accumulation
 *     is float32 (float64 for TD_F64).
 *   - stream is a cudaStream_t (NULL = legacy default stream). Kernels are queued on it; nothing is synchronised.
 *   - Return 0 (TD_OK) on success. Otherwise a TD_ERR_* code and, when err is not NULL, a NUL-terminated message
 *     in err[0 .. err_len). Argument errors are detected before any launch; launch errors are read with
 *     cudaGetLastError before returning.
 *   - No entry point allocates device memory. td_project_forward takes a caller-provided workspace.
 */
#ifndef TINYDEFORM_H_
#define TINYDEFORM_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TD_API __attribute__((visibility("default")))
#else
#define TD_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum td_dtype { TD_F32 = 0, TD_F16 = 1, TD_BF16 = 2, TD_F64 = 3 };

enum td_status {
    TD_OK = 0,
    TD_ERR_ARG = 1,         /* a size, pointer or dtype violates the contract; nothing was launched */
    TD_ERR_CUDA = 2,        /* a CUDA runtime call or kernel launch failed */
    TD_ERR_WORKSPACE = 3    /* the workspace is NULL or smaller than the call's *_workspace_bytes() */
};

/* Limits of the operator contract (upstream csrc/ma_deform_fused.cu:27-28 and :241,:264). */
#define TD_MAX_LEVEL_POINTS 64   /* L * P per head */
#define TD_MAX_CHANNELS 8192     /* C for the fused order */

/*
 * Fused order: gather the bilinear corners of full C-wide memory rows per (batch, query, head), then project the
 * weighted sum with that head's value_weight rows, plus value_bias * (sum of in-map corner weights).
 * Replaces upstream fused_forward (csrc/ma_deform_fused.cu:291-325), called from
 * marearts_tinydeform/__init__.py:74-76.
 *   memory [B, N, C]; value_weight [HD, C]; value_bias [HD] or NULL; sampling_locations [B, Q, H, L, P, 2];
 *   attention_weights [B, Q, H, L, P]; out [B, Q, HD] (written).  HD % H == 0, D = HD / H.
 */
TD_API int td_fused_forward(int dtype, const void* memory, const void* value_weight, const void* value_bias,
                     const int64_t* spatial_shapes, const int64_t* level_start_index,
                     const void* sampling_locations, const void* attention_weights, void* out,
                     int64_t B, int64_t Q, int64_t N, int64_t C, int64_t H, int64_t HD, int64_t L, int64_t P,
                     void* stream, char* err, size_t err_len);

/*
 * Project order, sampling half: sample an already projected value [B, N, HD] (bias included).
 * Replaces upstream sample_forward (csrc/ma_deform_fused.cu:327-350), called from
 * marearts_tinydeform/__init__.py:78-79.  heads must equal H.
 */
TD_API int td_sample_forward(int dtype, const void* value, int64_t heads, const int64_t* spatial_shapes,
                      const int64_t* level_start_index, const void* sampling_locations,
                      const void* attention_weights, void* out,
                      int64_t B, int64_t Q, int64_t N, int64_t HD, int64_t H, int64_t L, int64_t P,
                      void* stream, char* err, size_t err_len);

/*
 * Project order, projection half: value = memory @ value_weight^T + value_bias, written either as [B, N, HD]
 * (head_major = 0, the nn.Linear layout) or head-major [B, H, N, D] (head_major = 1, the layout the sampler of
 * td_project_forward reads). Replaces the F.linear call of upstream marearts_tinydeform/__init__.py:77.
 */
TD_API int td_value_proj(int dtype, const void* memory, const void* value_weight, const void* value_bias, void* value,
                  int64_t B, int64_t N, int64_t C, int64_t H, int64_t HD, int head_major,
                  void* stream, char* err, size_t err_len);

/*
 * y = x @ weight^T + bias for row-major x [M, K], weight [Nout, K], bias [Nout] or NULL, y [M, Nout]: the
 * tensor-core projection kernel, launched with programmatic dependent launch so that its set-up overlaps the kernel
 * before it in the stream (it waits for that kernel before reading x). For the decoder's output_proj right after
 * ma_deform_attn (the nn.Linear callers apply to its result, upstream README.md:11); no counterpart in upstream.
 */
TD_API int td_linear(int dtype, const void* x, const void* weight, const void* bias, void* y, int64_t M, int64_t K,
                     int64_t Nout, void* stream, char* err, size_t err_len);

/*
 * The producer of sampling_locations / attention_weights in the multi-scale deformable attention layer (Deformable-
 * DETR's MSDeformAttn, RT-DETR's decoder), from proj = query @ [W_offsets; W_attention]^T + [b_offsets; b_attention]
 * (td_linear): proj [B * Q, 3 * H * L * P], each row the 2 * H * L * P offsets (head, level, point, x/y) then the
 * H * L * P attention logits (head, level * point). Per (b, q, h): attention_weights = softmax over the L * P logits;
 * sampling_locations = ref[b, q, l] + offset / (w_l, h_l) for reference_points [B, Q, L, 2] (ref_dim 2), or
 * ref.xy + offset / P * ref.wh * 0.5 for reference boxes [B, Q, L, 4] (ref_dim 4). Writes sampling_locations
 * [B, Q, H, L, P, 2] and attention_weights [B, Q, H, L, P]. Upstream takes both as inputs and has no producer.
 */
TD_API int td_sampling_producer(int dtype, const void* proj, const void* reference_points, int ref_dim,
                                const int64_t* spatial_shapes, void* sampling_locations, void* attention_weights,
                                int64_t B, int64_t Q, int64_t H, int64_t L, int64_t P, void* stream, char* err,
                                size_t err_len);

/*
 * Backward of td_sampling_producer: from grad_locations [B, Q, H, L, P, 2] and grad_weights [B, Q, H, L, P] (either
 * may be NULL, meaning zero) and the forward's inputs, writes grad_proj [B, Q, 3 * H * L * P] (same layout as proj:
 * offset gradients, then logit gradients through the softmax) and, unless grad_reference_points is NULL,
 * grad_reference_points [B, Q, L, ref_dim] (summed over heads and points, in a fixed order: no atomics). One CTA
 * per (batch, query), a warp per head. Launched with programmatic dependent launch. No counterpart in upstream (no producer, no
 * backward); the definition followed is the producer's own (Deformable-DETR's MSDeformAttn forward).
 */
TD_API int td_sampling_producer_backward(int dtype, const void* proj, const void* reference_points, int ref_dim,
                                         const int64_t* spatial_shapes, const void* grad_locations,
                                         const void* grad_weights, void* grad_proj, void* grad_reference_points,
                                         int64_t B, int64_t Q, int64_t H, int64_t L, int64_t P, void* stream,
                                         char* err, size_t err_len);

/*
 * td_project_forward_masked followed by the decoder's output_proj in the same call: out [B, Q, C_out] =
 * attention @ output_weight^T + output_bias, output_weight [C_out, HD] (nn.Linear), output_bias [C_out] or NULL;
 * the output GEMM (the projection kernel, as td_linear) is queued right behind the sampler with programmatic
 * dependent launch. output_weight NULL: exactly td_project_forward_masked. Workspace:
 * td_project_ex_workspace_bytes(dtype, B, Q, N, HD, output_weight != NULL) bytes (the projected value, plus the
 * attention result). No upstream counterpart (upstream's callers apply output_proj themselves, README.md:11).
 */
TD_API size_t td_project_ex_workspace_bytes(int dtype, int64_t B, int64_t Q, int64_t N, int64_t HD, int output_proj);
TD_API int td_project_forward_ex(int dtype, const void* memory, const void* value_weight, const void* value_bias,
                                 const int64_t* spatial_shapes, const int64_t* level_start_index,
                                 const void* sampling_locations, const void* attention_weights,
                                 const uint8_t* value_padding_mask, const void* output_weight,
                                 const void* output_bias, int64_t C_out, void* out, int64_t B, int64_t Q, int64_t N,
                                 int64_t C, int64_t H, int64_t HD, int64_t L, int64_t P, void* workspace,
                                 size_t workspace_bytes, void* stream, char* err, size_t err_len);

/*
 * Backward of the sampling half (upstream's CUDA operator is inference only; this is the derivative of its
 * reference, reference.py:29-40, as autograd computes it through grid_sample): given grad_out [B, Q, H * D] for
 * out = sample(value, sampling_locations, attention_weights), writes
 *   grad_value [B, N, H * D] -- float32, float64 for TD_F64 -- zeroed here, then accumulated with atomics (the sum
 *                                order, and so the last bits, vary from run to run),
 *   grad_sampling_locations [B, Q, H, L, P, 2] and grad_attention_weights [B, Q, H, L, P] in dtype.
 * value is addressed through element strides as in td_sample_strided (the head-major [B, H, N, D] layout the
 * projection writes: s_img = H * N * D, s_tok = D, s_head = N * D); value_padding_mask [B, N] or NULL (a padded
 * token's value counts as zero and receives no gradient). The gradients of memory, value_weight and value_bias
 * follow from grad_value by two plain GEMMs and a column sum (the caller's).
 */
TD_API int td_sample_backward(int dtype, const void* value, int64_t s_img, int64_t s_tok, int64_t s_head,
                              const int64_t* spatial_shapes, const int64_t* level_start_index,
                              const void* sampling_locations, const void* attention_weights,
                              const uint8_t* value_padding_mask, const void* grad_out, void* grad_value,
                              void* grad_sampling_locations, void* grad_attention_weights, int64_t B, int64_t Q,
                              int64_t N, int64_t H, int64_t D, int64_t L, int64_t P, void* stream, char* err,
                              size_t err_len);

/*
 * One pass over td_sample_backward's float32 grad_value [rows, HD] (rows = B * N): rounds it into
 * grad_value_dtype [rows, HD] (float16 / bfloat16; ignored for TD_F32, where the accumulator is used as it is) and
 * writes its column sums -- the value bias gradient -- into grad_bias (float32 [HD], zeroed here; NULL: skipped).
 * HD a multiple of 4, at most 1024; 16-byte aligned buffers.
 */
TD_API int td_grad_value_finish(int dtype, const float* grad_value, void* grad_value_dtype, float* grad_bias,
                                int64_t rows, int64_t HD, void* stream, char* err, size_t err_len);

/*
 * One multi-scale deformable attention layer of a DETR-style decoder (Deformable-DETR's MSDeformAttn forward, the
 * caller of upstream's operator), in one call:
 *   proj = query [B, Q, Cq] @ sampling_weight^T + sampling_bias       sampling_weight = [W_offsets; W_attention],
 *                                                                     [3 * H * L * P, Cq] (td_sampling_producer)
 *   locations, weights = the producer of td_sampling_producer on proj and reference_points [B, Q, L, ref_dim]
 *   attn = ma_deform_attn(memory [B, N, C], value_weight [HD, C], value_bias, ...)  [B, Q, HD], with the optional
 *          value padding mask [B, N] of td_project_forward_masked
 *   out  = attn @ output_weight^T + output_bias  [B, Q, C_out] when output_weight is not NULL, else out = attn.
 * order TD_ORDER_PROJECT: two launches -- the value and query projections in one tensor-core launch (when both fit
 * it and share C; else two), then the sampler whose corner prologue runs the producer, so locations and weights
 * never reach memory; TD_ORDER_FUSED: query projection, producer, the fused gather-then-project kernel. Plus the
 * output projection. Intermediates live in `workspace` of at least
 * td_layer_workspace_bytes() bytes (same arguments; output_proj = output_weight != NULL). No counterpart in upstream,
 * which implements only the operator.
 */
enum td_order { TD_ORDER_PROJECT = 0, TD_ORDER_FUSED = 1 };
TD_API size_t td_layer_workspace_bytes(int dtype, int order, int64_t B, int64_t Q, int64_t N, int64_t H, int64_t HD,
                                       int64_t L, int64_t P, int output_proj);
TD_API int td_layer_forward(int dtype, int order, const void* query, int64_t Cq, const void* reference_points,
                            int ref_dim, const void* sampling_weight, const void* sampling_bias, const void* memory,
                            const void* value_weight, const void* value_bias, const uint8_t* value_padding_mask,
                            const int64_t* spatial_shapes, const int64_t* level_start_index,
                            const void* output_weight, const void* output_bias, int64_t C_out, void* out, int64_t B,
                            int64_t Q, int64_t N, int64_t C, int64_t H, int64_t HD, int64_t L, int64_t P,
                            void* workspace, size_t workspace_bytes, void* stream, char* err, size_t err_len);

/*
 * Sampling of a projected value at explicit element strides: value element (b, token, head, d) is at
 * b * s_img + token * s_tok + head * s_head + d. td_sample_forward is the case (N*HD, HD, D); the head-major value
 * td_project_forward samples is (H*N*D, D, N*D). Generalises upstream sample_forward
 * (csrc/ma_deform_fused.cu:327-350) so each half of the project order can be run and timed on its own.
 */
TD_API int td_sample_strided(int dtype, const void* value, int64_t s_img, int64_t s_tok, int64_t s_head,
                             const int64_t* spatial_shapes, const int64_t* level_start_index,
                             const void* sampling_locations, const void* attention_weights, void* out,
                             int64_t B, int64_t Q, int64_t N, int64_t H, int64_t D, int64_t L, int64_t P,
                             void* stream, char* err, size_t err_len);

/* Bytes of device workspace td_project_forward needs (the projected value, head-major, plus alignment slack). */
TD_API size_t td_project_workspace_bytes(int dtype, int64_t B, int64_t N, int64_t HD);

/*
 * Project order, whole: td_value_proj (head-major) into the workspace, then the per-head sampler on it.
 * Replaces upstream marearts_tinydeform/__init__.py:77-79 (F.linear + _C.sample_forward).
 */
TD_API int td_project_forward(int dtype, const void* memory, const void* value_weight, const void* value_bias,
                       const int64_t* spatial_shapes, const int64_t* level_start_index,
                       const void* sampling_locations, const void* attention_weights, void* out,
                       int64_t B, int64_t Q, int64_t N, int64_t C, int64_t H, int64_t HD, int64_t L, int64_t P,
                       void* workspace, size_t workspace_bytes, void* stream, char* err, size_t err_len);

/*
 * Both orders with a value padding mask. No counterpart in upstream (whose value has no mask); the semantics are
 * Deformable-DETR's input_padding_mask: value = memory @ W^T + b, then value[b, n, :] = 0 wherever
 * value_padding_mask[b * N + n] != 0. A padded token thus contributes nothing to the output, its bias included: its
 * bilinear corners count as outside the map. value_padding_mask is a device array of B * N bytes (torch.bool
 * layout), or NULL for no mask (the unmasked entry points above).
 */
TD_API int td_fused_forward_masked(int dtype, const void* memory, const void* value_weight, const void* value_bias,
                            const int64_t* spatial_shapes, const int64_t* level_start_index,
                            const void* sampling_locations, const void* attention_weights,
                            const uint8_t* value_padding_mask, void* out, int64_t B, int64_t Q, int64_t N, int64_t C,
                            int64_t H, int64_t HD, int64_t L, int64_t P, void* stream, char* err, size_t err_len);
TD_API int td_project_forward_masked(int dtype, const void* memory, const void* value_weight, const void* value_bias,
                              const int64_t* spatial_shapes, const int64_t* level_start_index,
                              const void* sampling_locations, const void* attention_weights,
                              const uint8_t* value_padding_mask, void* out, int64_t B, int64_t Q, int64_t N,
                              int64_t C, int64_t H, int64_t HD, int64_t L, int64_t P, void* workspace,
                              size_t workspace_bytes, void* stream, char* err, size_t err_len);

/*
 * Project order with no caller-provided workspace and no allocation at all. No counterpart in upstream.
 *
 * For callers that cannot allocate device memory on the call path: inference plugins run inside a host framework
 * that owns all device memory (and forbids cudaMalloc in enqueue), real-time loops where cudaMalloc's implicit
 * device synchronisation is not acceptable, and plain C hosts with no caching allocator to borrow a workspace from.
 * The projected value lives instead in one file-scope device array of TD_NOALLOC_SCRATCH_BYTES that every GPU which
 * loads this library holds until the process exits. Requests whose value (td_project_workspace_bytes) exceeds it
 * are rejected with TD_ERR_WORKSPACE and a message naming both sizes; the RT-DETR 640x640 layer (B=1, N=8400,
 * H*D=256) needs 4.3 MB in 16-bit types and 8.6 MB in float32.
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress) with that device current;
 * make that first call before any stream capture on the device. A first call made while its stream is capturing
 * is refused with TD_ERR_CUDA (nothing is launched or recorded); a failed lookup is not remembered, so a later call
 * tries again. Arguments are checked before the lookup. The array is shared by all calls and keeps the last call's
 * contents; it is fully rewritten before it is read, so nothing needs clearing. Calls whose work overlaps on the
 * GPU (other streams, other threads) race on it: serialise them.
 */
#define TD_NOALLOC_SCRATCH_BYTES ((size_t)16 << 20)
TD_API int td_project_forward_noalloc(int dtype, const void* memory, const void* value_weight, const void* value_bias,
                                      const int64_t* spatial_shapes, const int64_t* level_start_index,
                                      const void* sampling_locations, const void* attention_weights, void* out,
                                      int64_t B, int64_t Q, int64_t N, int64_t C, int64_t H, int64_t HD, int64_t L,
                                      int64_t P, void* stream, char* err, size_t err_len);

/*
 * The GEMMs of a linear layer's backward, for the training path (no counterpart in upstream, whose operator is
 * inference only, marearts_tinydeform/__init__.py:67-71; they replace the cuBLAS GEMMs torch's autograd would run for
 * nn.Linear). For y = x @ weight^T (+ bias), x [M, K], weight [Nout, K] and grad_out = dL/dy [M, Nout]:
 *   td_linear_grad_input:  grad_input [M, K] = grad_out @ weight
 *   td_linear_grad_weight: grad_weight [Nout, K] = grad_out^T @ x, summed over all M rows; grad_bias [Nout] (the
 *                          column sums of grad_out) when grad_bias is not NULL. Outputs in the input dtype.
 * In the operator's backward x is memory, weight value_weight and grad_out the gradient of the projected value.
 * float16 / bfloat16 run on tcgen05 tensor cores (float32 accumulation) when every row is 16-byte aligned
 * (Nout, K multiples of 8); float32 / float64 and other shapes on CUDA cores. On the tensor cores the weight
 * gradient splits the M rows over CTAs, each storing its float32 partial tile, and a second kernel sums the partials
 * in a fixed order (bitwise reproducible); the bias gradient's column sums and the CUDA-core weight gradient add
 * partial sums atomically, so their last bits may vary between runs.
 * td_linear_grad_weight needs td_linear_grad_workspace_bytes(dtype, Nout, K) bytes of workspace (the split partials,
 * at most 256 x 64 KB; 0 for float32 and float64, whose sums accumulate in the outputs themselves).
 */
TD_API size_t td_linear_grad_workspace_bytes(int dtype, int64_t Nout, int64_t K);
TD_API int td_linear_grad_input(int dtype, const void* grad_out, const void* weight, void* grad_input, int64_t M,
                                int64_t Nout, int64_t K, void* stream, char* err, size_t err_len);
TD_API int td_linear_grad_weight(int dtype, const void* grad_out, const void* input, void* grad_weight,
                                 void* grad_bias, int64_t M, int64_t Nout, int64_t K, void* workspace,
                                 size_t workspace_bytes, void* stream, char* err, size_t err_len);

/*
 * Test of the bounded waits (no counterpart in upstream): every wait of the tensor-core kernels on a TMA or MMA
 * completion gives up after about a second, records a code in the device error word (td_device_error) and lets the
 * kernel free its tensor memory and exit, so that a stuck pipeline ends in an error status rather than a hung GPU.
 * This call makes the NEXT float16 / bfloat16 tensor-core launch of td_linear_grad_input / td_linear_grad_weight
 * starve its own pipeline -- its TMA producers issue nothing, so no copy or MMA is ever in flight -- and give up
 * each wait after spin_limit_cycles (1 .. 2e9) instead: its output is left unwritten, the error word holds the code
 * of the first wait that ran out, and later launches are ordinary. Returns TD_ERR_ARG for a limit out of range.
 */
TD_API int td_test_starve_next_grad_gemm(long long spin_limit_cycles);

/*
 * Measurement kernel (no counterpart in upstream): reads `visits` pseudo-random rows of row_bytes (a power of two,
 * 16..512; 32..512 with wide = 1, which uses 32-byte loads) from buf ([rows, row_bytes], 16- or 32-byte aligned)
 * with every SM, the way the sampler reads corner rows, and writes one 16-byte word per thread into sink
 * (sink_bytes >= grid * 256 * 16). visits must be a multiple of grid * 8 * (32 / lanes per row) * (wide ? 4 : 8);
 * the message of a rejected call names the multiple. Timing it over an L2-resident buffer gives the L2 random-row
 * gather rate the gather kernels' roofline is measured against (bench.py --l2-peak).
 */
TD_API int td_probe_row_gather(const void* buf, int64_t rows, int row_bytes, int wide, int64_t visits, unsigned seed,
                               void* sink, size_t sink_bytes, int grid, void* stream, char* err, size_t err_len);

/*
 * Batch sharding with the output all-gather fused into the sampler (no upstream counterpart: upstream has no
 * distributed code; this replaces the project order's separate all-gather collective). One process per GPU; every
 * rank holds a gathered output buffer [B_global, Q, H * D] and a control block, allocated here and mapped into every
 * other rank through CUDA IPC (the handles travel over the caller's own host collective):
 *   td_peer_buffer_alloc  cudaMalloc'd, zeroed buffer and its IPC handle (TD_IPC_HANDLE_BYTES bytes);
 *   td_peer_buffer_open   a peer's buffer from its handle (peer access enabled lazily); closed by
 *   td_peer_buffer_close  (opened = 1 for a peer's mapping, 0 for this process's own allocation).
 * td_project_forward_peer computes this rank's B images (global images first_image .. first_image + B - 1) in the
 * project order and stores every output row into all `world` buffers (outputs[r] = rank r's buffer as mapped in
 * this process, controls[r] likewise its control block of TD_PEER_CTRL_BYTES bytes, zeroed at allocation); a one-warp
 * kernel behind it signals every peer once the rows are stored and waits (bounded, about one second; a peer that
 * never signals sets code TD_DEVERR_PEER_WAIT in td_device_error) until every peer has signalled this call. After it,
 * the buffer holds every rank's rows. Every rank must make the same sequence of calls (a rank with no images passes
 * B = 0 and still signals). Epochs are kept in the control blocks on the device, so a captured CUDA graph replays
 * correctly. A peer may write the next call's rows as soon as this rank's wait has finished: consume the buffer
 * before the next call, or alternate two buffer sets. Shapes: D * element size of 16 * 2^k bytes up to 512; 1-8
 * ranks; workspace td_project_workspace_bytes(dtype, B, N, HD).
 */
#define TD_IPC_HANDLE_BYTES 64
#define TD_PEER_CTRL_BYTES 64
#define TD_DEVERR_PEER_WAIT 5
TD_API int td_peer_buffer_alloc(size_t bytes, void** ptr, void* ipc_handle, char* err, size_t err_len);
TD_API int td_peer_buffer_open(const void* ipc_handle, void** ptr, char* err, size_t err_len);
TD_API int td_peer_buffer_close(void* ptr, int opened, char* err, size_t err_len);
TD_API int td_project_forward_peer(int dtype, const void* memory, const void* value_weight, const void* value_bias,
                                   const int64_t* spatial_shapes, const int64_t* level_start_index,
                                   const void* sampling_locations, const void* attention_weights,
                                   const uint8_t* value_padding_mask, int64_t B, int64_t Q, int64_t N, int64_t C,
                                   int64_t H, int64_t HD, int64_t L, int64_t P, int64_t first_image, int world,
                                   int rank, void* const* outputs, void* const* controls, void* workspace,
                                   size_t workspace_bytes, void* stream, char* err, size_t err_len);
/* Test only: the peer wait alone on one control block, with a wait limit of limit_cycles clock cycles (a test makes
 * it run out on one GPU by naming a peer that never signals). */
TD_API int td_test_peer_wait(void* control, int world, int rank, long long limit_cycles, void* stream, char* err,
                             size_t err_len);

/*
 * Kernel policy for every later call in this process: TD_POLICY_BEST (default) uses the tcgen05 tensor-core
 * kernels wherever the shapes allow; TD_POLICY_CUDA_CORES keeps every call on the CUDA-core kernels (parity tests
 * run both). No counterpart in upstream, which has only CUDA-core kernels. Returns the previous policy.
 */
enum td_policy { TD_POLICY_BEST = 0, TD_POLICY_CUDA_CORES = 1 };
TD_API int td_set_kernel_policy(int policy);

/*
 * How calls that apply output_proj in the project order (td_project_forward_ex, td_layer_forward) run it, for
 * every later call in this process. TD_OUTPROJ_AUTO (default): in the sampler's own kernel (thread-block clusters
 * of 8 CTAs share the attention rows over distributed shared memory and split Wo's columns) while that kernel's grid
 * is one wave (B * Q * H / 8 <= 3 CTAs per SM: 444 queries at 8 heads on B200), chained as a separate GEMM above
 * that. TD_OUTPROJ_CHAINED: always chained.
 * TD_OUTPROJ_CLUSTER: in the sampler's kernel wherever its conditions hold (H dividing 8, H * D * element size of
 * 512 bytes, C_out <= 256, 16-byte aligned Wo and value rows of 16 * 2^k bytes up to 512), else chained.
 * Results agree within the dtype's rounding either way. No counterpart in upstream, which has no output_proj
 * (its README lists fusing it as future work, README.md:11). Returns the previous plan, or -1 for an unknown plan.
 */
enum td_outproj_plan { TD_OUTPROJ_AUTO = 0, TD_OUTPROJ_CHAINED = 1, TD_OUTPROJ_CLUSTER = 2 };
TD_API int td_set_output_proj_plan(int plan);

/*
 * Reads the library's device error word on the current device (0 = no error), and clears it when `clear` is set.
 * The tensor-core kernels bound every wait; a wait that gives up (about one second) stores a non-zero code here
 * instead of hanging. Synchronises with the device. No counterpart in upstream.
 */
TD_API int td_device_error(int clear, unsigned int* code, char* err, size_t err_len);

/* Device facts used by the auto picker and the bench: SM count and compute capability of `device`. */
TD_API int td_device_info(int device, int* sm_count, int* cc_major, int* cc_minor, char* err, size_t err_len);

/* Number of kernels this library has queued since it was loaded (host-side counter; graph replays not counted). */
TD_API uint64_t td_launch_count(void);

/* Library version string, e.g. "0.1.1+b200". */
TD_API const char* td_version(void);

#ifdef __cplusplus
}
#endif

#endif /* TINYDEFORM_H_ */
