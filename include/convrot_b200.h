/*
 * C ABI of the B200 (sm_100a) ConvRot W4A4 library, libconvrot_b200.so.
 *
 * Drop-in for the HIP library of 0xDELUXA/ComfyUI-INT4-ConvRot-RDNA4
 * (_int4/int4_gemm.hip). Paths below are relative to that project.
 *
 * Conventions (same as the reference exports, _int4/int4_gemm.hip:627-741):
 *   - all pointers are device pointers; the caller allocates every output;
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream);
 *   - launches are asynchronous and nothing synchronises inside a call;
 *   - return 0 on success, -1 when a shape/pointer precondition fails (nothing
 *     is launched; ck_convrot_last_error() explains), otherwise a cudaError_t.
 *
 * Layouts (the reference codec, _int4/_codec.py:19-36):
 *   packed int4 matrix [rows, K/2] int8, row-major; byte j of a row holds
 *   column 2j in its low nibble and column 2j+1 in its high nibble, both two's
 *   complement. Scales are float32, one per row (tokens) / output channel.
 */
#ifndef CONVROT_B200_H
#define CONVROT_B200_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Fused ConvRot rotation + row-wise int4 quantization + packing.
 * Replaces ck_convrot_quant_int4 (_int4/int4_gemm.hip:650-660), bound by
 * convrot_quant_int4 (_int4/hip_loader.py:74-92).
 *   x        [M, K] activations, in_dtype 0 = f32, 1 = bf16, 2 = f16
 *   qout     [M, K/2] int8 packed codes
 *   scaleout [M] f32 row scales
 * G in {16, 64, 256}, K % G == 0, K % 16 == 0. Quantizer arithmetic follows
 * the eager path (_int4/eager.py:112-120) in the activation dtype. */
int ck_convrot_quant_int4(const void* x, int in_dtype, void* qout, void* scaleout,
                          int M, int K, int G, void* stream);

/* Row-wise int4 quantization + packing of an already rotated activation
 * (rotation skipped). Replaces quantize_signed_int4_rowwise
 * (_int4/eager.py:112-120) for device tensors; same arguments as above minus G. */
int ck_int4_quant_rowwise(const void* x, int in_dtype, void* qout, void* scaleout,
                          int M, int K, void* stream);

/* out[m, n] = ((float(D[m, n]) * xscale[m]) * wscale[n]) + bias[n],
 * D = exact int32 sum_k X[m, k] * W[n, k] over packed codes.
 * Replaces ck_int4_convrot_gemm (_int4/int4_gemm.hip:711-741), bound by
 * int4_convrot_gemm (_int4/hip_loader.py:158-207).
 *   Xp [M, K/2], Wp [N, K/2] packed int8 (16-byte aligned)
 *   xscale [M], wscale [N], bias [N] or NULL: f32
 *   out [M, N], out_dtype 0 = f32, 1 = bf16
 * K % 32 == 0 and K <= 65536. */
int ck_int4_convrot_gemm(const void* Xp, const void* Wp, const void* xscale, const void* wscale,
                         const void* bias, void* out, int M, int N, int K, int out_dtype,
                         void* stream);

/* Workspace bytes that ck_convrot_w4a4_linear needs for M rows of K: the
 * activation codes and the row scales [M] f32, each from a 256-byte boundary.
 * The codes take [M, K/2] bytes (packed) below 129 rows and [M, K] bytes (one
 * per code, for the A8 form below) from 129 rows on. No reference counterpart. */
size_t ck_convrot_w4a4_linear_workspace_size(int M, int K);

/* The whole W4A4 linear in one call: rotate + quantize x (as
 * ck_convrot_quant_int4) into `workspace`, then
 * out = ((float(D) * xs[m]) * wscale[n]) + bias[n] (as ck_int4_convrot_gemm).
 * Replaces the two-call sequence of the reference's Python convrot_w4a4_linear
 * (_int4/__init__.py:94-135: convrot_quant_int4 then int4_convrot_gemm); no
 * single HIP export does both. Differences from calling the two exports:
 *   - bias is read in its own dtype, bias_dtype 0 = f32, 1 = bf16, 2 = f16
 *     (widening is exact, so results equal an fp32-converted bias);
 *   - the GEMM launch is a programmatic dependent of the quantizer launch;
 *   - bf16 x with 129+ rows, K % 256 == 0 and G in {64, 256} takes the A8
 *     form: codes written one per byte, then ck_int4_convrot_gemm_a8 (same
 *     accumulators, same output bits).
 *   x [M, K] in_dtype (0 f32, 1 bf16, 2 f16); Wp [N, K/2]; wscale [N] f32;
 *   out [M, N] out_dtype (0 f32, 1 bf16); G in {16, 64, 256}, K % G == 0,
 *   K % 32 == 0; workspace 256-byte aligned, at least
 *   ck_convrot_w4a4_linear_workspace_size(M, K) bytes, no initial contents
 *   needed; two calls in flight at once need two workspaces. */
int ck_convrot_w4a4_linear(const void* x, int in_dtype, const void* Wp, const void* wscale,
                           const void* bias, int bias_dtype, void* out, int out_dtype,
                           int M, int N, int K, int G, void* workspace, size_t workspace_bytes,
                           void* stream);

/* ck_convrot_w4a4_linear for callers that cannot allocate device memory (a
 * host framework that owns every device buffer through its own arena and only
 * hands this library inputs and outputs, a plugin ABI with plain pointers and
 * no allocator): the same arguments minus the workspace, which is replaced by
 * a static 128 MiB device array per device, placed when the library's no-alloc
 * module loads on that device. The entry itself allocates nothing. No
 * reference counterpart: the reference always allocates its intermediates
 * with torch.
 *   - limit: ck_convrot_w4a4_linear_workspace_size(M, K) <= 134217728 bytes
 *     (e.g. M = 18432 rows at K = 12288); larger sizes return -1 before any
 *     CUDA call, with the reason in ck_convrot_last_error();
 *   - nothing in the scratch has to start at zero (it is fully rewritten by
 *     each call before it is read);
 *   - one scratch per device: calls that may overlap in time (other streams,
 *     other host threads) race on it; calls on one stream are ordered and safe;
 *   - the first call on each device does the setup (a cudaGetSymbolAddress
 *     with that device current), and so does the first call after that
 *     device's primary context was reset: make it before any stream capture;
 *   - with lazy module loading (the default) only processes that call this
 *     entry hold the 128 MiB; with CUDA_MODULE_LOADING=EAGER every process
 *     that loads the library holds it on each device it uses. */
int ck_convrot_w4a4_linear_noalloc(const void* x, int in_dtype, const void* Wp, const void* wscale,
                                   const void* bias, int bias_dtype, void* out, int out_dtype,
                                   int M, int N, int K, int G, void* stream);

/* ck_int4_convrot_gemm plus a fused Dynamic-LoRA side path:
 *   out[m, n] = (((float(D) * xscale[m]) * wscale[n]) + bias[n]) + lora_scale * L[m, n],
 *   L = lora_t[m, :] . lora_b[n, :]  (fp16 operands, fp32 tensor-core accumulation).
 * lora_t = x A^T [M, rank] and lora_b = B [N, rank] are fp16 row-major (the
 * reference's adapter dtype, int4_ops.py:165-167); rank a
 * multiple of 8 in [8, 64]; bias in bias_dtype as for ck_convrot_w4a4_linear.
 * Replaces the unfused per-adapter `out + v.h(x, out)`
 * of the node's forward (int4_ops.py:181-192, :383); no HIP export counterpart. */
int ck_int4_convrot_gemm_lora(const void* Xp, const void* Wp, const void* xscale, const void* wscale,
                              const void* bias, int bias_dtype, void* out, int M, int N, int K,
                              int out_dtype, const void* lora_t, const void* lora_b, int rank,
                              float lora_scale, void* stream);

/* ck_int4_convrot_gemm_lora on int8 operands X [M, K], W [N, K] (the W8A8 tier,
 * or int4 codes sign-extended by ck_int4_unpack / ck_convrot_quant_int4_unpacked,
 * which give the same D and so the same output bits); same epilogue, arguments
 * and return codes. No reference counterpart (the reference's int8 layers add
 * the LoRA side path after the GEMM, int4_ops.py:371-383). */
int ck_int8_convrot_gemm_lora(const void* X, const void* W, const void* xscale, const void* wscale,
                              const void* bias, int bias_dtype, void* out, int M, int N, int K,
                              int out_dtype, const void* lora_t, const void* lora_b, int rank,
                              float lora_scale, void* stream);

/* accum[m, n] += (float(D[m, n]) * xscale[m]) * wscale[n] into a caller-zeroed
 * f32 [M, N] buffer. Replaces ck_int4_convrot_gemm_splitk
 * (_int4/int4_gemm.hip:634-645). The reference splits K and adds float
 * partials with atomics; here D is reduced in int32 first, so the result is
 * deterministic. `nsplit` (>= 1) is accepted for ABI compatibility. */
int ck_int4_convrot_gemm_splitk(const void* Xp, const void* Wp, const void* xscale,
                                const void* wscale, void* accum, int M, int N, int K,
                                int nsplit, void* stream);

/* Raw exact int32 accumulators acc[M, N] = sum_k X[m, k] * W[n, k].
 * No reference counterpart as an export: the reference computes these inside
 * its GEMM (_int4/int4_gemm.hip:204-232); exposed for bit-exact parity checks. */
int ck_int4_gemm_s32(const void* Xp, const void* Wp, void* acc, int M, int N, int K, void* stream);

/* W8A8 tier (the int8 middle tier of mixed precision).
 *
 * Fused ConvRot rotation + row-wise int8 quantization, codes not packed.
 * Replaces ck_convrot_quant_int8 (_int4/int4_gemm.hip:664-672), bound by
 * convrot_quant_int8 (_int4/hip_loader.py:95-113); the quantizer arithmetic is
 * the eager one in the activation dtype (_int4/int8_eager.py:22-27: scale =
 * dtype(absmax / 127), q = rint(dtype(x / scale)) clamped to +-127).
 *   x [M, K] (in_dtype must be 1 = bf16), qout [M, K] int8 (16-byte aligned),
 *   scaleout [M] f32; G in {64, 256} and K % 256 == 0 (other dtypes, G = 16 or
 *   ragged K return -1: the caller keeps its torch path, as the reference's
 *   Python layer does for shapes its kernel does not take). */
int ck_convrot_quant_int8(const void* x, int in_dtype, void* qout, void* scaleout,
                          int M, int K, int G, void* stream);

/* out[m, n] = ((float(D[m, n]) * xscale[m]) * wscale[n]) + bias[n],
 * D = exact int32 sum_k X[m, k] * W[n, k] of int8 values.
 * Replaces ck_int8_convrot_gemm (_int4/int4_gemm.hip:676-705), bound by
 * int8_convrot_gemm (_int4/hip_loader.py:116-150).
 *   X [M, K], W [N, K] int8 (16-byte aligned), xscale [M], wscale [N], bias [N]
 *   or NULL: f32; out [M, N], out_dtype 0 = f32, 1 = bf16; K % 16 == 0. */
int ck_int8_convrot_gemm(const void* X, const void* W, const void* xscale, const void* wscale,
                         const void* bias, void* out, int M, int N, int K, int out_dtype,
                         void* stream);

/* Raw exact int32 accumulators of the int8 product (no reference export; for
 * parity checks, like ck_int4_gemm_s32). */
int ck_int8_gemm_s32(const void* X, const void* W, void* acc, int M, int N, int K, void* stream);

/* The rotation fused into the producer of x (no reference counterpart; the
 * reference quantizes what the model's LayerNorm/modulation kernels wrote):
 * each bf16 row is normalised and modulated as a Flux block does before its
 * QKV or MLP-up projection,
 *   y = bf16(bf16(bf16(1 + mod_scale[k]) * xn) + mod_shift[k]),
 *   xn = bf16((x - mean) * rstd), rstd = 1 / sqrt(var + eps)
 * (LayerNorm without affine, biased variance; fp32 statistics in a fixed order:
 * lane l of a warp sums elements l, l + 32, ... then an xor butterfly of the 32
 * lane sums), then rotated and quantized exactly as ck_convrot_quant_int4 would
 * quantize y. y never goes to memory. mod_scale / mod_shift: bf16 [K], one
 * vector for all M rows (call once per batch item), NULL = zeros (plain
 * LayerNorm). bf16 x only; G in {64, 256}; K % 256 == 0, K <= 6144.
 * unpacked = 1 writes one sign-extended int8 per code ([M, K], the A8 form's
 * operand), 0 packed codes ([M, K/2]). */
int ck_convrot_quant_int4_lnmod(const void* x, const void* mod_scale, const void* mod_shift, float eps,
                                void* qout, void* scaleout, int M, int K, int G, int unpacked, void* stream);

/* ck_convrot_w4a4_linear of the modulated LayerNorm of x (as above), one pass
 * over x: out = y @ W^T + bias with the int4 path's arithmetic; same workspace
 * size rule (ck_convrot_w4a4_linear_workspace_size). */
int ck_convrot_w4a4_linear_lnmod(const void* x, const void* mod_scale, const void* mod_shift, float eps,
                                 const void* Wp, const void* wscale, const void* bias, int bias_dtype,
                                 void* out, int out_dtype, int M, int N, int K, int G, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* Column-split linear over peer memory (no reference counterpart: the
 * reference runs on one device). P ranks (one process per GPU) each own N/P
 * weight rows; every rank's GEMM stores its column block straight into every
 * rank's [M, ldo] output through peer mappings over NVLink, then
 * ck_peer_barrier tells each rank that all blocks have landed in its output.
 *
 * ck_peer_buffer_alloc: cudaMalloc of `bytes` (zeroed) and its 64-byte CUDA IPC
 * handle; ck_peer_buffer_open maps another process's buffer from its handle
 * (ck_peer_buffer_close unmaps it); ck_peer_buffer_free frees an own buffer. */
int ck_peer_buffer_alloc(size_t bytes, void** ptr, void* ipc_handle);
int ck_peer_buffer_open(const void* ipc_handle, void** ptr);
int ck_peer_buffer_close(void* ptr);
int ck_peer_buffer_free(void* ptr);

/* ck_int4_convrot_gemm_a8 (packed weights, int8 activation codes, optional
 * LoRA side path; same D, epilogue and output bits) storing its [M, N] result
 * as columns col0 .. col0 + N of the [M, ldo] row-major matrices outs[0 ..
 * nouts) (1 to 8 pointers, any of them peer mappings; ldo and col0 multiples
 * of 8). Plain stores, no multicast. */
int ck_int4_convrot_gemm_a8_peers(const void* X8, const void* Wp, const void* xscale, const void* wscale,
                                  const void* bias, int bias_dtype, void* const* outs, int nouts,
                                  int ldo, int col0, int M, int N, int K, int out_dtype,
                                  const void* lora_t, const void* lora_b, int rank,
                                  float lora_scale, void* stream);

/* Barrier of nranks (<= 8) ranks after their peer stores: flags[p] is rank p's
 * flag array (int32 [nranks], this process's mapping of it; zero when
 * allocated), counter a 4-byte device word of this rank (zero at the start,
 * advanced by every call, so the call can sit in a CUDA graph). Rank `rank`
 * writes this call's epoch into slot `rank` of every rank's flags (release,
 * system scope, after a system fence) and waits until every slot of its own
 * flags has reached it. A wait longer than timeout_ns records status 6
 * (ck_convrot_device_status) and returns instead of hanging. Every rank must
 * make the same sequence of calls. */
int ck_peer_barrier(void* const* flags, int nranks, int rank, void* counter, long long timeout_ns, void* stream);

/* Copy columns [offset, offset + width) (bytes) of `rows` rows of pitch
 * pitch_bytes from src to the same place in each of dsts[0 .. ndst) (peer
 * mappings allowed): one 2D copy per destination on `stream`, carried by the
 * copy engines over NVLink, so no SM time is taken from kernels running beside
 * it. The column-split linear sends each rank's block to its peers this way. */
int ck_peer_copy_columns(void* const* dsts, int ndst, const void* src, long long pitch_bytes,
                         long long offset_bytes, long long width_bytes, long long rows, void* stream);

/* Dynamic-LoRA down projection T = fp16(x) . down^T (no HIP export counterpart;
 * replaces the fp16 matmul the node's adapter runs on x, int4_ops.py:181-192,
 * with the adapters in fp16 as int4_ops.py:165-167 prepares them):
 *   x [M, K] in in_dtype (1 = bf16, converted to fp16 element by element with
 *   round to nearest even, as a cast does; 2 = f16), down [R, K] f16,
 *   t [M, R] f16 out; K % 8 == 0, R a multiple of 8 in [8, 64], all 16-byte
 *   aligned. fp32 accumulation on the tensor cores, one rounding to fp16; the
 *   summation order is fixed, so results repeat bit for bit. t is the lora_t
 *   operand of the fused LoRA GEMMs. */
int ck_lora_down(const void* x, int in_dtype, const void* down, void* t, int M, int K, int R, void* stream);

/* The int4 GEMM on int8 activation codes (A8 form; no reference counterpart):
 *   X8 [M, K] int8, one sign-extended code per byte (ck_convrot_quant_int4_unpacked),
 *   Wp [N, K/2] packed int4 weights (the reference codec), both 16-byte aligned;
 *   xscale [M], wscale [N] f32; bias [N] or NULL in bias_dtype (0 f32, 1 bf16, 2 f16);
 *   out [M, N], out_dtype 0 = f32, 1 = bf16, 3 = int32 exact accumulators D
 *   (scales and bias ignored); K % 128 == 0, K <= 65536.
 * Optional Dynamic-LoRA side path as ck_int4_convrot_gemm_lora (lora_t, lora_b
 * fp16 [M, rank] / [N, rank], rank a multiple of 8 in [8, 64]; both NULL: none).
 * The weights stay packed in HBM and are expanded on chip (into tensor memory
 * for grids of 74+ output tiles without LoRA, else in shared memory); the
 * activations go to the tensor cores as loaded. Same D, epilogue and output
 * bits as the packed-code GEMM. */
int ck_int4_convrot_gemm_a8(const void* X8, const void* Wp, const void* xscale, const void* wscale,
                            const void* bias, int bias_dtype, void* out, int M, int N, int K,
                            int out_dtype, const void* lora_t, const void* lora_b, int rank,
                            float lora_scale, void* stream);

/* Unpacked-code path (no reference counterpart). With both operands as one
 * sign-extended int8 per int4 code, sum_k x_k w_k is the int8 tensor-core product
 * over the same K: bit-identical results to the packed path on the faster int8
 * pipeline, at twice the bytes for the operands. */

/* packed [rows, K/2] -> codes [rows, K] int8 (column order kept, nibbles
 * sign-extended); both 16-byte aligned, K % 32 == 0. Run once per weight. */
int ck_int4_unpack(const void* packed, void* codes, long long rows, int K, void* stream);

/* ck_convrot_quant_int4 with unpacked output: codes [M, K] int8, scale [M] f32.
 * bf16 rows of whole 256-column tiles, G in {64, 256}; -1 otherwise. */
int ck_convrot_quant_int4_unpacked(const void* x, int in_dtype, void* qout, void* scaleout,
                                   int M, int K, int G, void* stream);

/* Workspace of ck_convrot_w4a4_linear_unpacked: align256(M * K) + align256(4 * M). */
size_t ck_convrot_w4a4_linear_unpacked_workspace_size(int M, int K);

/* ck_convrot_w4a4_linear with the weight given as unpacked codes Wcodes [N, K]
 * int8 (from ck_int4_unpack): the quantizer writes unpacked activation codes to
 * the workspace and the int8 pair GEMM (double-buffered accumulators) forms the
 * exact products; same epilogue, same results. Same argument rules as
 * ck_convrot_w4a4_linear plus those of ck_convrot_quant_int4_unpacked. */
int ck_convrot_w4a4_linear_unpacked(const void* x, int in_dtype, const void* Wcodes, const void* wscale,
                                    const void* bias, int bias_dtype, void* out, int out_dtype,
                                    int M, int N, int K, int G, void* workspace, size_t workspace_bytes,
                                    void* stream);

/* Reads and clears the device status word that kernels set when a bounded
 * wait gives up (0 = ok). Synchronises `stream`. No reference counterpart:
 * the reference has no device-side timeouts. */
int ck_convrot_device_status(void* stream, int* status);

/* Failure-path self test: launches one thread that waits on an mbarrier nothing
 * arrives on, with the bounded wait every pipeline wait uses, cut to limit_ns
 * (0 < limit_ns <= 1e8). It gives up, records status 5 (read and cleared by
 * ck_convrot_device_status) and returns, leaving the context usable. No
 * reference counterpart: it exercises the timeout path without faulting a GPU. */
int ck_convrot_selftest_wait_timeout(long long limit_ns, void* stream);

/* Human-readable reason for the last -1 returned on this host thread. */
const char* ck_convrot_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* CONVROT_B200_H */
