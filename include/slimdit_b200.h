/*
 * slimdit_b200 — C ABI of the B200 (sm_100a) convrot W8A8 linear and weight converter.
 *
 * Conventions for every entry point:
 *   - All array arguments are device pointers owned by the caller; shapes are element
 *     counts; matrices are row-major. `stream` is a cudaStream_t passed as void* (NULL =
 *     legacy default stream). Calls are stream-ordered and do not synchronise.
 *   - Return 0 on success or a negative SLIM_ERR_* code; no exception crosses the ABI.
 *     slim_last_error() returns the message of the calling thread's last failure.
 *   - Device pointers must be 16-byte aligned; rows are contiguous (pitch = K).
 *   - Kernel-side waits are bounded; slim_device_error() reports (and clears) a wait that
 *     ran out.
 *
 * Rotation orders (`order`):
 *   SLIM_ORDER_REFERENCE reproduces the reference's fp32 summation order of
 *     `np.matmul(grouped, H.T)` (slimdit/hadamard.py:56-58, numpy 2.3 + OpenBLAS 0.3.30
 *     on x86-64), so codes and scales equal slimdit.int8.quantize_convrot_weight's bit for
 *     bit. For rows of 5..64 groups (K = 1280..16384) with rot_out NULL it runs at the cost
 *     of the fast transform (a certified butterfly: the reference's sequential chains are
 *     evaluated only for the few outputs whose code or whose row maximum they can change);
 *     otherwise compute-bound (~256 fp32 FMAs per element). The linears below quantise their
 *     activations in this order.
 *   SLIM_ORDER_BUTTERFLY is the radix-4 fast Hadamard transform alone (memory-bound): a few
 *     codes per million and ~4 % of row scales differ from the reference's (counted by the
 *     tests and the benchmark).
 */
#ifndef SLIMDIT_B200_H_
#define SLIMDIT_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SLIM_ABI_VERSION 1

enum slim_status {
  SLIM_OK = 0,
  SLIM_ERR_SHAPE = -1,       /* bad or unsupported shape */
  SLIM_ERR_ALIGN = -2,       /* pointer or pitch not 16-byte aligned */
  SLIM_ERR_GROUP = -3,       /* group size other than 256, or K % 256 != 0 */
  SLIM_ERR_ARCH = -4,        /* device is not sm_100 */
  SLIM_ERR_CUDA = -5,        /* CUDA runtime error (see slim_last_error) */
  SLIM_ERR_DTYPE = -6,       /* unsupported dtype / order / epilogue code */
  SLIM_ERR_NULL = -7         /* required pointer is NULL */
};

enum slim_dtype { SLIM_F32 = 0, SLIM_BF16 = 1, SLIM_F16 = 2 };
enum slim_order { SLIM_ORDER_REFERENCE = 0, SLIM_ORDER_BUTTERFLY = 1 };
/* SLIM_EPI_SWIGLU (INT8 GEMM only): the weight's rows are interleaved per 256-row tile, 128
 * "up" rows then the 128 matching "gate" rows (slim_swiglu_interleave order); the output
 * has N/2 columns, out[m, t*128 + i] = bf16(up * bf16(silu(gate))) with up and gate the bf16
 * linear outputs of rows 256t + i and 256t + 128 + i: ComfyUI's swiglu ([up; gate],
 * slimdit/mapping.py:96-97) on the bf16 output of the fc1 linear, fused. N % 256 == 0. */
enum slim_epilogue { SLIM_EPI_SCALE_BIAS = 0, SLIM_EPI_GELU_TANH = 1, SLIM_EPI_SWIGLU = 2 };

/* ABI version (SLIM_ABI_VERSION). */
int slim_version(void);

/* Copies the calling thread's last error message (NUL-terminated) into buf.
 * Returns the message length. */
int slim_last_error(char* buf, size_t len);

/* Synchronises the current device, stores the device error word (0 = none; see
 * slim_ptx.cuh DeviceError) in *code and clears it. */
int slim_device_error(unsigned int* code);

/* Number of kernels this library has launched since it was loaded. */
uint64_t slim_launch_count(void);

/* Group-wise rotation out = W @ H^T over groups of 256 input features, fp32 result.
 * Replaces slimdit.hadamard.rotate(weight, h, group_size) (slimdit/hadamard.py:45-58).
 * x: [rows, K] of `dtype`; out: fp32 [rows, K]. */
int slim_rotate_f32(const void* x, int dtype, int64_t rows, int64_t K, int group, int order,
                    float* out, void* stream);

/* Rotation fused with per-row symmetric INT8 quantisation:
 *   scale[r] = max(absmax_r / 127, 1e-30),  q = clip(rint(rot / scale), -128, 127).
 * Replaces slimdit.int8.quantize_convrot_weight (slimdit/int8.py:39-52) for weights and the
 * per-token activation quantisation inside the runtime's int8_linear
 * (tools/bench_int8.py:65-68), the same per-row math applied to token rows.
 * q: int8 [rows, K]; scale: fp32 [rows]; rot_out: optional fp32 [rows, K] copy of the
 * rotated values (NULL to skip). BUTTERFLY requires K <= 16384. */
int slim_rotate_quant_i8(const void* x, int dtype, int64_t rows, int64_t K, int group,
                         int order, int8_t* q, float* scale, float* rot_out, void* stream);

/* Quantisation stage alone on already-rotated fp32 rows (slimdit/int8.py:49-51). */
int slim_quantize_rows_i8(const float* rotated, int64_t rows, int64_t K, int8_t* q,
                          float* scale, void* stream);

/* out = (q * scale) @ H^T in the reference order.
 * Replaces slimdit.int8.dequantize_convrot_weight (slimdit/int8.py:55-61). */
int slim_dequant_i8(const int8_t* q, const float* scale, int64_t rows, int64_t K, int group,
                    float* out, void* stream);

/* out[m,n] = bf16(float(sum_k a[m,k]*b[n,k]) * (sa[m]*sb[n]) + bias[n]), optionally
 * followed by GELU-tanh (SLIM_EPI_GELU_TANH: applied to the bf16-rounded linear output,
 * result rounded to bf16). a: int8 [M,K]; b: int8 [N,K]; sa: fp32 [M]; sb: fp32 [N];
 * bias: bf16 [N] or NULL; out: bf16 [M,N]; acc_dbg: int32 [M,N] or NULL (raw
 * accumulators). Requires K % 16 == 0 and N % 8 == 0.
 * The int8 GEMM + dequant inside the runtime's int8_linear (tools/bench_int8.py:65-68;
 * math at slimdit/int8.py:9-11). */
int slim_gemm_i8(const int8_t* a, const int8_t* b, const float* sa, const float* sb,
                 const void* bias, void* out, int32_t* acc_dbg, int64_t M, int64_t N,
                 int64_t K, int epilogue, void* stream);

/* The convrot W8A8 linear: rotate + quantise the bf16/f16/f32 activation x [M,K] per
 * token (REFERENCE order) into the caller's workspaces xq_ws (int8 [M,K]) and sx_ws
 * (fp32 [M]), then slim_gemm_i8 against the pre-rotated weight codes qw [N,K] with row
 * scales sw [N]. Drop-in for comfy_kitchen.int8_linear(x, qweight, wscales, convrot=True,
 * convrot_groupsize=256, out_dtype=bf16) (tools/bench_int8.py:65-68). */
int slim_int8_linear(const void* x, int x_dtype, const int8_t* qw, const float* sw,
                     const void* bias, void* out, int8_t* xq_ws, float* sx_ws, int64_t M,
                     int64_t N, int64_t K, int group, int epilogue, void* stream);

/* The DiT FFN: out[M, K] = down(requant(act(up(x)))) on the device, stream-ordered, into the
 * caller's workspaces. act = SLIM_EPI_GELU_TANH: w_up int8 [F, K] (the GELU-tanh FFN);
 * act = SLIM_EPI_SWIGLU: w_up int8 [2F, K] with its rows interleaved per 256 (128 up rows,
 * then the matching 128 gate rows; slimdit.ops.swiglu_interleave), the MiniMax-H3 FFN
 * (slimdit/mapping.py:96-101). The up-projection's epilogue applies the activation to its
 * bf16 outputs, h is rotated and requantised per token, then the down-projection w_down int8
 * [K, F]. s_up/s_down fp32 row scales, b_up/b_down bf16 biases or NULL. Workspaces: xq_ws
 * int8 [M, K], sx_ws fp32 [M], h_ws bf16 [M, F], hq_ws int8 [M, F], sh_ws fp32 [M]. */
int slim_ffn_i8(const void* x, int x_dtype, const int8_t* w_up, const float* s_up,
                const void* b_up, const int8_t* w_down, const float* s_down,
                const void* b_down, void* out, int8_t* xq_ws, float* sx_ws, void* h_ws,
                int8_t* hq_ws, float* sh_ws, int64_t M, int64_t K, int64_t F, int act,
                void* stream);

/* The convrot linear without caller workspaces, for callers that cannot allocate device
 * memory: code running inside a host framework that owns the device memory pool (a plugin
 * given only its inputs and outputs), or on a path where an allocation would synchronise
 * or fail under a memory cap. No counterpart exists in the reference (its runtime op
 * allocates through torch).
 * Same arguments and result as slim_int8_linear, minus xq_ws/sx_ws: the activation codes
 * and scales go to one 32 MiB array compiled into the library, which every GPU that loads
 * the library holds until exit. Limit: round_up(M*K, 256) + 4*M <= 32 MiB (e.g. 6400
 * tokens at K = 5120); larger calls return SLIM_ERR_SHAPE. The first call on a device (and
 * again the first in another CUDA context of it) looks up the array's device address
 * (cudaGetSymbolAddress); make it before any stream capture. All calls share the array:
 * calls that overlap on the GPU race. Allocates nothing (no cudaMalloc/cudaFree). */
int slim_int8_linear_noalloc(const void* x, int x_dtype, const int8_t* qw, const float* sw,
                             const void* bias, void* out, int64_t M, int64_t N, int64_t K,
                             int group, int epilogue, void* stream);

/* Allocates `bytes` of device memory on the current device that other processes can map
 * (cudaMalloc + cudaIpcGetMemHandle): *ptr receives the buffer, ipc_handle (64 bytes) its
 * CUDA IPC handle for slim_peer_open in the other processes. Free with
 * slim_peer_buffer_free after every process has closed its mapping. */
int slim_peer_buffer_alloc(size_t bytes, void** ptr, void* ipc_handle);
int slim_peer_buffer_free(void* ptr);

/* Maps another process's device allocation into this process on the current device (CUDA
 * IPC, peer access over NVLink enabled on first use): ipc_handle is the 64-byte
 * cudaIpcMemHandle_t of the allocation, offset the byte offset of the buffer inside it.
 * *ptr receives the mapped buffer address. Plain peer mapping: no multicast object. */
int slim_peer_open(const void* ipc_handle, int64_t offset, void** ptr);

/* Unmaps a buffer opened by slim_peer_open (ptr and offset as returned and given there). */
int slim_peer_close(void* ptr, int64_t offset);

/* Stream-ordered 2-D copy of `height` rows of `width` bytes between any two device buffers
 * of this process (local or peer-mapped; the copy engines move it over NVLink). */
int slim_copy_2d(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t width,
                 int64_t height, void* stream);

/* The convrot linear with its output columns split over the GPUs of a node: this GPU
 * computes y[:, c0:c0+N] for its weight rows qw/sw/bias [N, K] (x [M, K] replicated) and the
 * GEMM epilogue stores every output tile into each of the n_outs buffers `outs` (host array of
 * device pointers: this GPU's output and the other GPUs' outputs mapped into this process,
 * e.g. symmetric memory over NVLink), each already offset to column c0, rows ldo elements
 * apart. The all-gather of the reference plan (an NCCL collective after the GEMM) happens
 * inside the GEMM, tile by tile. The caller synchronises the GPUs after the call (all ranks'
 * stores done) before reading. n_outs <= 8. No reference counterpart: the reference runs
 * one GPU; this is the optional output-column split of the B200 plan. */
int slim_int8_linear_colsplit(const void* x, int x_dtype, const int8_t* qw, const float* sw,
                              const void* bias, void* const* outs, int n_outs, int64_t ldo,
                              int8_t* xq_ws, float* sx_ws, int64_t M, int64_t N, int64_t K,
                              int group, int epilogue, void* stream);

/* ---------------------------------------------------------------- NVFP4
 * Format of slimdit/nvfp4.py:3-8: E2M1 codes packed two per byte, high nibble first (element
 * 2i in the high nibble, 2i+1 in the low one; activations too, so that both operands of the
 * FP4 GEMM share the order), one UE4M3 scale per 16 consecutive elements along K stored in the cuBLAS 128x4
 * tiled layout (scale (r, c) of a [R, C = K/16] matrix at byte
 * ((r/128)*(C/4) + c/4)*512 + (r%32)*16 + ((r%128)/32)*4 + c%4), and an fp32 global scale
 * gs = amax / (448 * 6). Block scale = e4m3(min(fl(fl(block_amax / 6) / gs), 448)); codes =
 * E2M1 round-half-even of fl(x / fl(gs * block_scale)). All sizes need K % 64 == 0 and
 * K <= 16384. */

/* Weight packing with one global scale per tensor. Replaces
 * slimdit.nvfp4.quantize_nvfp4_weight (slimdit/nvfp4.py:72-87; the reference delegates the
 * arithmetic to comfy_kitchen's TensorCoreNVFP4Layout.quantize).
 * w: [rows, K] of `dtype`, rows % 128 == 0; q: uint8 [rows, K/2]; block_scale: uint8
 * [rows, K/16]; tensor_scale: one fp32 in device memory (weight_scale_2). */
int slim_nvfp4_pack(const void* w, int dtype, int64_t rows, int64_t K, uint8_t* q,
                    uint8_t* block_scale, float* tensor_scale, void* stream);

/* Activation quantisation for the NVFP4 linear: one global scale per token row
 * (row_scale fp32 [rows]), optionally after the group-256 Hadamard rotation in the
 * butterfly order (rotate != 0; K % 256 == 0). q: uint8 [rows, K/2]; block_scale: uint8
 * [round_up(rows, 128), K/16] (padding rows get zero scales). The input side of the NVFP4
 * runtime linear that consumes slimdit/nvfp4.py's format (the NVFP4 up-projection). */
int slim_quant_nvfp4_act(const void* x, int dtype, int64_t rows, int64_t K, int rotate,
                         uint8_t* q, uint8_t* block_scale, float* row_scale, void* stream);

/* out[r, k] = code * fl(scale * block_scale) in fp32 (scale[0] for the tensor, or
 * scale[r] when per_row). out may be NULL when err is given; err (fp64[2] in device
 * memory, accumulated into, not cleared) receives sum (out - x)^2 and sum x^2 against the
 * original x of x_dtype: the round-trip error of slimdit.nvfp4.quantize_nvfp4_with_error
 * (slimdit/nvfp4.py:90-105). */
int slim_nvfp4_dequant(const uint8_t* q, const uint8_t* block_scale, const float* scale,
                       int per_row, int64_t rows, int64_t K, float* out, const void* x,
                       int x_dtype, double* err, void* stream);

/* out[m,n] = bf16(acc * (a_scale[m] * b_scale[0]) + bias[n]) (optionally GELU-tanh),
 * acc = sum_k (a[m,k] * a_sf) * (b[n,k] * b_sf) accumulated in fp32 by the block-scaled
 * tensor cores (tcgen05 kind::mxf4nvf4). a: [M, K/2], a_sf: [round_up(M,128), K/16];
 * b: [N, K/2] with N % 128 == 0, b_sf: [N, K/16]; acc_dbg: fp32 [M, N] or NULL.
 * The FP4 GEMM of the NVFP4 runtime linear (the reference measures comfy_kitchen's,
 * docs/DEV_NOTES.md:204-206). */
int slim_gemm_nvfp4(const uint8_t* a, const uint8_t* a_sf, const float* a_scale,
                    const uint8_t* b, const uint8_t* b_sf, const float* b_scale,
                    const void* bias, void* out, float* acc_dbg, int64_t M, int64_t N,
                    int64_t K, int epilogue, void* stream);

/* The NVFP4 linear: slim_quant_nvfp4_act of x [M,K] into the caller's workspaces
 * (xq_ws uint8 [M, K/2], xsf_ws uint8 [round_up(M,128), K/16], xs_ws fp32 [M]), then
 * slim_gemm_nvfp4 against the packed weight (qw, w_sf, w_scale). */
int slim_nvfp4_linear(const void* x, int x_dtype, const uint8_t* qw, const uint8_t* w_sf,
                      const float* w_scale, const void* bias, void* out, uint8_t* xq_ws,
                      uint8_t* xsf_ws, float* xs_ws, int64_t M, int64_t N, int64_t K,
                      int rotate, int epilogue, void* stream);

/* ---------------------------------------------------------------- verification
 * Relative-L2 building blocks of tools/verify_checkpoint.py (compare_reference /
 * compare_official, tools/verify_checkpoint.py:81-152), reduced in fp64 on the GPU. Both add
 * sum (a - b)^2 to out2[0] and sum b^2 to out2[1] (device fp64[2], not cleared). */

/* INT8 rows in the rotated basis, a = fl32(qa * sa[row]), b = fl32(qb * sb[row]): the
 * load_value(rotated=True) comparison (tools/verify_checkpoint.py:71-75). K % 16 == 0. */
int slim_rel_l2_int8(const int8_t* qa, const float* sa, const int8_t* qb, const float* sb,
                     int64_t rows, int64_t K, double* out2, void* stream);

/* Two n-element tensors of SLIM_F32/BF16/F16, compared as fp32 values. */
int slim_rel_l2(const void* a, int a_dtype, const void* b, int b_dtype, int64_t n,
                double* out2, void* stream);

/* ---------------------------------------------------------------- attention
 * In-place INT8/FP8 flash attention on the DiT's packed qkv buffer: the reference's
 * TritonAttnOverride._run (comfyui/ComfyUI-SlimDiT/attention_triton.py:265-299) and its
 * kernels quant_int8_rows, tensor_amax, quant_fp8_global and flash_int8 (:79-174).
 * Head dim 128 only. seq_pad is seq rounded up to a multiple of 128 (or larger, a multiple of
 * 128); per-head scale rows are [heads, seq_pad] fp32 and their padding is written as 0. */

/* Bytes of the workspace slim_attn_packed needs for (seq, heads, dim). */
int slim_attn_workspace_bytes(int64_t seq, int heads, int dim, uint64_t* bytes);

/* q and k rows of the bf16 buffer qkv (row pitch row_stride elements; q at column q_offset,
 * k at k_offset): rotate != 0 applies the +-1 Sylvester Hadamard over each (token, head)
 * row first; scale = max(amax, 1e-8) / 127, code = clip(floor(x / scale + 0.5), -127, 127)
 * (quant_int8_rows, attention_triton.py:79-102). q, k: int8 [seq, heads*dim];
 * q_scale_t, k_scale_t: fp32 [heads, seq_pad]. */
int slim_attn_quant_qk(const void* qkv, int64_t seq, int heads, int dim, int64_t row_stride,
                       int64_t q_offset, int64_t k_offset, int rotate, int8_t* q,
                       float* q_scale_t, int8_t* k, float* k_scale_t, int64_t seq_pad,
                       void* stream);

/* v rows of qkv (column v_offset) -> *v_amax = max|v| (device fp32 scalar) and
 * v_t = E4M3(v / max(amax / 448, 1e-8)), transposed per head: uint8 [heads, dim, seq_pad],
 * zero padded (tensor_amax + quant_fp8_global, attention_triton.py:104-129, 283-287). */
int slim_attn_quant_v(const void* qkv, int64_t seq, int heads, int dim, int64_t row_stride,
                      int64_t v_offset, uint8_t* v_t, int64_t seq_pad, float* v_amax,
                      void* stream);

/* The two halves of slim_attn_quant_v, for callers that split the heads over several GPUs:
 * the V scale is global over all heads (attention_triton.py:283-286), so each GPU computes the
 * amax of its own heads, the maxima are reduced (one float), and every GPU quantises its heads
 * with the common amax. slim_attn_v_amax writes max|v| of the given heads to *v_amax;
 * slim_attn_quant_v_scaled quantises with the given *v_amax. */
int slim_attn_v_amax(const void* qkv, int64_t seq, int heads, int dim, int64_t row_stride,
                     int64_t v_offset, float* v_amax, void* stream);
int slim_attn_quant_v_scaled(const void* qkv, int64_t seq, int heads, int dim,
                             int64_t row_stride, int64_t v_offset, uint8_t* v_t,
                             int64_t seq_pad, const float* v_amax, void* stream);

/* out[seq, ldo] bf16 (head h at columns [h*dim, h*dim+dim)) = softmax attention of the
 * quantised q/k/v above with logits s * q_scale * k_scale * attn_scale, P rounded to E4M3
 * for both P V and the row sum (flash_int8, attention_triton.py:131-174). */
int slim_attn_int8(const int8_t* q, const float* q_scale_t, const int8_t* k,
                   const float* k_scale_t, const uint8_t* v_t, const float* v_amax,
                   float attn_scale, int64_t seq, int heads, int dim, int64_t seq_pad,
                   void* out, int64_t ldo, void* stream);

/* The whole override on a packed [seq, 3*heads*dim] bf16 buffer: the three calls above with
 * attn_scale = dim^-0.5 / (rotate ? dim : 1); out bf16 [seq, heads*dim]. */
int slim_attn_packed(const void* qkv, int64_t seq, int heads, int dim, int rotate, void* out,
                     void* workspace, uint64_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SLIMDIT_B200_H_ */
