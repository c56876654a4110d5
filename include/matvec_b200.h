/* Entry points of libmatvec_b200.so beyond the reference's six (include/matvec_fpga.h). None of these has a
 * counterpart in driver/matvec_fpga.h; the unchanged reference hosts never call them. They take CUDA device
 * pointers and a CUDA stream of the current device (as void *; NULL = CUDA's default stream), run
 * asynchronously and return 0, or -1 with the reason in mvb_last_error() (and on stderr).
 *
 * The arithmetic of every matvec here is the reference's (qwen.c:436-456, runq.c:430-458): int32 group sums,
 * p = ((float)isum * wscale) * xscale, groups added in order. Outputs are bit-identical to the reference C.
 */
#ifndef MATVEC_B200_H
#define MATVEC_B200_H
#include <stddef.h>
#include <stdint.h>
#include "matvec_fpga.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Text of the last error raised by any entry point of this library ("" if none). */
const char *mvb_last_error(void);

/* fpga_matvec4's computation on device pointers (the qwen path, hls4/matvec4.h:1-21): w (d*n*wbits/8 bytes),
 * ws (d*n/32 fp16), xq (n int8), xs (n/32 fp32) -> out (d fp32). wbits 4 or 8, n % 32 == 0, n <= 8192, d >= 1;
 * w and xq 16-byte aligned, ws 2-byte, xs and out 4-byte aligned. */
int mvb_matvec4(const void *w, const void *ws, const void *xq, const void *xs, float *out, int n, int d, int wbits,
                void *stream);

/* fpga_matvec's computation on device pointers (the runq path, hls/matvec.h:1-19): wq (d*n int8), ws (d*n/gs
 * fp32), xq (n int8), xs (n/gs fp32) -> out (d fp32). gs 32 or 64, n % gs == 0, n <= 8192, d >= 1;
 * wq and xq 16-byte aligned, ws/xs/out 4-byte aligned. */
int mvb_matvec(const void *wq, const void *ws, const void *xq, const void *xs, float *out, int n, int d, int gs,
               void *stream);

/* mvb_matvec4 with the activation quantization fused into the kernel's prologue: x is n fp32 values, quantized
 * per group of 32 exactly like qwen.c's quantize() (qwen.c:355-364) inside every CTA. x 16-byte aligned. */
int mvb_qmatvec4(const void *w, const void *ws, const float *x, float *out, int n, int d, int wbits, void *stream);

/* mvb_matvec with runq.c's quantize() (runq.c:244-270) fused into the prologue. x 16-byte aligned. */
int mvb_qmatvec(const void *wq, const void *ws, const float *x, float *out, int n, int d, int gs, void *stream);

/* Rows per CTA tile that the launchers pick for a d x n matrix (exposed for the benchmark's accounting). */
int mvb_rows_per_tile(int n, int d);


/* ---- Device-resident decode (the reference's token loops, qwen/qwen.c:490-712 and runq/runq.c:477-1026, on
 * the device) ----
 * The whole forward step (embedding, per-layer rmsnorm/quantize/matvecs/attention/SwiGLU, head, greedy argmax)
 * runs on the current CUDA device as one captured CUDA graph, every matvec being this library's kernel. Token
 * and position live in device memory, so a generation is one graph launch per position with no host work.
 * Two loaders make a decoder handle: mvb_qwen_load (a .qwb model, qwen.c's arithmetic) and mvb_runq_load (a runq
 * version 2 checkpoint, runq.c's arithmetic). Every mvb_qwen_* call below takes either handle; "head" means
 * qwen.c's trimmed head or runq.c's classifier (head_k = vocab_size rows, the row being the token id).
 * All calls below are synchronous except mvb_qwen_rewind and mvb_qwen_launch, and wait at most
 * MATVEC_TIMEOUT_S (default 5 s) plus 10 ms per position. */

/* Uploads a .qwb image (the whole file's bytes, layout of tools/gguf2qwb.py:5-15) to the current device and
 * captures the decode step; ctx is the KV-cache length (clipped to the header's max_seq_len like qwen.c:325,
 * at most 8192). Returns a handle, or NULL with the reason in mvb_last_error(). */
void *mvb_qwen_load(const void *qwb_image, size_t bytes, int ctx);

/* mvb_qwen_load of the .qwb file at `path`, mapped read-only and uploaded from the page cache (no host copy). */
void *mvb_qwen_load_file(const char *path, int ctx);

/* Loads a runq version 2 checkpoint (the whole file's bytes, runq.c:318-357: int8 weights with fp32 scales,
 * shared or separate classifier) to the current device, each tensor in its own aligned slot, and captures the
 * decode step with runq.c's arithmetic (its quantize, rmsnorm eps 1e-5, interleaved RoPE, no biases, greedy
 * argmax over the classifier). Needs group size 32 or 64 (the two runq.c's FPGA build accepts) and head size 32,
 * 48 or 64. ctx is clipped to the header's seq_len. Returns a decoder handle, or NULL with the reason. */
void *mvb_runq_load(const void *checkpoint, size_t bytes, int ctx);

/* mvb_runq_load of the checkpoint file at `path`, mapped read-only (no host copy). */
void *mvb_runq_load_file(const char *path, int ctx);

/* out[0..8] = dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, head rows in use (head_k, or
 * vocab_size with a full head), ctx, kernels per step. */
int mvb_qwen_config(void *model, int *out);

/* on = 1: the head of a .qwb model becomes the full vocabulary. Qwen2 ties its output head to the token embedding,
 * so the Q8 embedding (vocab_size rows) serves as the head and its argmax row is the token id; on = 0: back to
 * the file's trimmed head_k-row head mapped through head_ids (qwen.c's). The trimmed head's logit i equals the
 * full head's logit head_ids[i] bit for bit. Recaptures the step; the KV cache and state are kept. A runq
 * handle's classifier is already full (on = 1 returns 0). No counterpart in the reference. 0, or -1. */
int mvb_qwen_full_head(void *model, int on);

/* The model's CUDA stream (every launch of the model is on it). */
void *mvb_qwen_stream(void *model);

/* One forward at `pos` with input `token` (qwen.c forward(), qwen.c:490-573); if logits is not NULL it receives
 * the head_k head logits. Returns the greedy head row (argmax, first of ties), or -1. */
int mvb_qwen_forward(void *model, int token, int pos, float *logits);

/* Feeds prompt[0 .. n-2] at positions 0 .. n-2 and leaves prompt[n-1] as the input of position n-1, like
 * qwen.c generate() before its first sampled token. The fed tokens run through the layers in batches of up to 256
 * with the tensor-core matmul (mvb_gemm4) and a batched causal attention, writing the KV-cache rows one decode
 * step per token would write, bit for bit (qwen.c computes the logits of prompt positions and discards them;
 * this skips the head there). A runq handle takes one decode step per fed token. 0, or -1. */
int mvb_qwen_prefill(void *model, const int *prompt, int n);

/* mvb_qwen_prefill's result reached one decode step per fed token (the reference's order of work). 0, or -1. */
int mvb_qwen_prefill_tokenwise(void *model, const int *prompt, int n);

/* Copies the KV-cache rows of positions 0 .. positions-1 of every layer into k and v (host arrays of n_layers *
 * positions * kv_dim floats, layer-major). 0, or -1. */
int mvb_qwen_cache(void *model, int positions, float *k, float *v);

/* Greedy decode of `steps` tokens from the current state; their token ids go to ids (host). Returns steps or -1. */
int mvb_qwen_decode(void *model, int steps, int *ids);

/* qwen.c generate() at -t 0 (qwen.c:669-712): prefill, then greedy ids into ids (host) until `steps`, a stop
 * token (<|im_end|>, <|endoftext|>, not copied) or a full context. Returns the number of ids, or -1. For a runq
 * handle this is runq.c generate() at -t 0 (runq.c:982-1026), whose stop token is BOS = 1. */
int mvb_qwen_generate(void *model, const int *prompt, int n_prompt, int steps, int *ids);

/* The same call under runq's name. runq.c's `-n steps` counts positions from 0, so it samples
 * steps - n_prompt + 1 tokens: pass that as `steps` here for the same run. */
int mvb_runq_generate(void *model, const int *prompt, int n_prompt, int steps, int *ids);

/* Sets the state to input `token` at position `pos` (positions below keep their KV cache), with n_prompt the
 * prompt length for the prompt/greedy switch (negative: no sampling). Asynchronous on the model's stream (the
 * state is copied from a pinned ring of 256 slots). Lets a benchmark repeat a decode from a filled cache. */
int mvb_qwen_rewind(void *model, int token, int pos, int n_prompt);

/* Runs one step with a CUDA event before every kernel and after the last (and no overlap between kernels),
 * writing each kernel's duration in ms to ms[0 .. count-1] (cap >= kernels per step). Returns the count or -1. */
int mvb_qwen_profile(void *model, float *ms, int cap);

/* Runs one step exactly as the captured graph runs it (programmatic dependent launch, no events between kernels),
 * with every kernel stamping the GPU's global timer: us[2k] = when kernel k's first CTA got past its wait for
 * kernel k - 1, us[2k + 1] = when its last CTA finished, in microseconds after the step's first kernel started
 * (cap >= 2 * kernels per step). us[2k + 1] - us[2k - 1] is kernel k's share of the step's critical path. The
 * state advances like a normal step. Returns the kernel count, or -1. */
int mvb_qwen_stamps(void *model, double *us, int cap);

/* Kernel k of the step: its kind ("embed", "qkv", "attention", "o_proj", "gate_up", "down", "final_norm",
 * "head", "next_token") into kind[kind_len], its layer (-1 outside the layers), and the bytes it must move at
 * position pos (weights, scales, activations, KV-cache rows). 0, or -1. */
int mvb_qwen_kernel_info(void *model, int k, int pos, char *kind, int kind_len, int *layer, double *bytes);

/* One forward at (token, pos) that also copies the residual stream x into trace (host,
 * (2 * n_layers + 1) * dim floats): after the embedding, then after each layer's attention and FFN blocks. */
int mvb_qwen_trace(void *model, int token, int pos, float *trace);

/* Enqueues `count` decode steps on the model's stream and returns without waiting. */
int mvb_qwen_launch(void *model, int count);

/* Frees the model's device memory, graph and stream. */
void mvb_qwen_free(void *model);

/* No counterpart in the reference. The decode's head path as one call that allocates nothing: rmsnorm of x with
 * norm_w and eps (qwen.c:337-344), quantize (qwen.c:355-364), then fpga_matvec4's computation of w/ws (d rows,
 * n columns, wbits 4 or 8) into out. All pointers are device pointers; the call is asynchronous on `stream`.
 * For callers that cannot allocate device memory while they run: hosts that size every device buffer once at
 * start-up (the reference's own qwen.c and runq.c carve all of theirs from one pre-sized pool), code on a
 * latency-critical path where cudaMalloc's implicit device-wide synchronization would stall other work, and code
 * inside a framework that owns the device allocator. Its scratch (the quantized activations) is a fixed device
 * array of 2,304 bytes that every GPU using the library holds until the process exits, so n is at most 2048
 * (larger n returns -1 with a message). The first call on each device looks up that array's address (again after
 * a cudaDeviceReset, whose next context holds a new copy of the array); make that first call before any stream
 * capture. Every pointer is checked (null; w 16-byte, ws 2-byte, x, norm_w and out 4-byte aligned) before anything
 * is launched, so a refused call changes nothing on the device. Every call overwrites the whole scratch it reads,
 * so nothing has to be cleared between calls, but all calls on a device share the one array: calls that can run
 * at the same time on one GPU (for example on two streams) race. Returns 0, or -1 with the reason in
 * mvb_last_error(). */
int mvb_norm_matvec4_static(const float *x, const float *norm_w, float eps, const void *w, const void *ws, float *out,
                            int n, int d, int wbits, void *stream);

/* The decode's expf on n device inputs x -> y (device pointers, asynchronous on `stream`): bit-identical to the
 * host C library's expf (the one qwen.c calls) on every float. The first call per process builds the table of
 * the library's non-correctly-rounded results (all host threads, a few seconds; cached in $MVB_CACHE_DIR, else
 * $XDG_CACHE_HOME/mvb or ~/.cache/mvb, in a file only this user may write, checked before use). entries/thresh (may be NULL) receive the table size and probe threshold. 0, or -1. */
int mvb_expf_eval(const float *x, float *y, int n, int *entries, float *thresh, void *stream);

/* ---- Batched prefill matmul on the tensor cores ----
 * No counterpart in the reference, which prefills token by token (qwen.c:674-681). m tokens through one matrix
 * at once: out[t * d + i] is fpga_matvec4's result for token t and row i, bit-identical to m separate matvecs.
 * w (d rows, n*wbits/8 bytes each, .qwb layout), ws (d * n/32 fp16), xq (m x n int8, token-major), xs (n/32 x ldx
 * fp32, group-major: xs[g * ldx + t] is token t's scale of group g; ldx >= m, ldx % 4 == 0), out (m x d fp32).
 * wbits 4 or 8, n % 32 == 0, n <= 8192; w, xq and xs 16-byte aligned. Device pointers, asynchronous on `stream`.
 * 0, or -1 with the reason in mvb_last_error(). */
int mvb_gemm4(const void *w, const void *ws, const void *xq, const float *xs, float *out, int n, int d, int m, int ldx,
              int wbits, void *stream);

/* Synchronizes `stream`; returns 0 if every GEMM kernel so far completed normally, or the code of the first
 * internal wait that gave up (the kernel then wrote no output), and clears it; -1 if the stream failed. */
int mvb_gemm_status(void *stream);

/* ---- Row-sharded matvec with the all-gather fused into the kernel (one process per GPU, NVLink peers) ----
 * No counterpart in the reference, which drives one board: this is fpga_matvec4 (driver/matvec_fpga.h:29-33)
 * for a matrix whose rows are split across `world` GPUs, rank r owning rows [r * rows, (r + 1) * rows). Each
 * rank's kernel stores its finished rows straight into every rank's gathered output over NVLink and signals
 * every rank's arrival counter; a bounded wait on the stream then holds back later work until all ranks' rows
 * have arrived. No NCCL call and no peer loads.
 *
 * Set-up: mvb_gather_create on every rank (fills `handle`, mvb_gather_handle_size() bytes, with this rank's
 * CUDA IPC handle), exchange the handles (any host channel), then mvb_gather_connect with all ranks' handles in
 * rank order. Every rank must then make the same sequence of mvb_gather_matvec4 calls with the same n. Every call
 * has the same launch arguments (the call number lives on the device), so a sequence of calls may be captured in a
 * CUDA graph and replayed on every rank. */
int mvb_gather_handle_size(void);
void *mvb_gather_create(int rank, int world, int rows, void *handle);  /* NULL on error */
/* The same with room for `tokens` tokens per call (mvb_gather_gemm4); mvb_gather_create holds one. */
void *mvb_gather_create_batch(int rank, int world, int rows, int tokens, void *handle);
int mvb_gather_connect(void *gather, const void *handles);            /* 0, or -1 */

/* This rank's shard (rows x n, wbits 4 or 8, .qwb layout; xq/xs the full activation vector) on `stream`. The
 * gathered output (rows * world fp32, rank-major) is mvb_gather_output's buffer once the stream reaches the
 * next operation. The output is double-buffered: read each call's output before the call after next. 0, or -1. */
int mvb_gather_matvec4(void *gather, const void *w, const void *ws, const void *xq, const void *xs, int n, int wbits,
                       void *stream);
/* Device pointer of the last completed call's gathered output (synchronous: reads the gather's call counter, which
 * the kernels keep on the device, so that calls replayed from a CUDA graph count too). */
float *mvb_gather_output(void *gather);

/* The batched form: m <= tokens tokens (xq m x n int8 token-major, xs n/32 x ldx fp32 group-major, as in
 * mvb_gemm4) through this rank's shard on the tensor cores; the gathered output is token-major, m x (rows * world)
 * fp32 (token t's row i of rank r at t * rows * world + r * rows + i). 0, or -1. */
int mvb_gather_gemm4(void *gather, const void *w, const void *ws, const void *xq, const float *xs, int n, int m,
                     int ldx, int wbits, void *stream);

/* 1 if a wait gave up (some rank's rows never arrived within 2 s), 0 if none did, -1 on error; synchronizes
 * `stream`. After a 1 the gather's counters no longer match: destroy it and create a new one on every rank. */
int mvb_gather_error(void *gather, void *stream);
void mvb_gather_destroy(void *gather);

#ifdef __cplusplus
}
#endif
#endif
