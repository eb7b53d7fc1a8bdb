/*
 * rwkv_b200.h — C ABI of the B200 (sm_100a) RWKV-7 packed-weight decode library.
 *
 * Drop-in boundary for the reference engine's native hot path.  The reference
 * binds one portable C file through ctypes (rwkv_ssd/native/lut2_gather.c,
 * loader rwkv_ssd/native/lut2_gather_loader.py:165-367); every entry point
 * below names the reference export or Python function it replaces.
 *
 * Conventions
 *  - Every pointer to weights, activations or outputs is a DEVICE pointer,
 *    except the `header` argument of rwkvb_packed_init (host bytes) and the
 *    host-side arrays of descriptors/pointers noted per function.
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *    Calls are asynchronous on that stream; outputs are ready when it is.
 *  - Every call returns an int status (RWKVB_OK = 0).  Invalid arguments or a
 *    malformed blob return RWKVB_EARG and launch nothing (the reference zero-
 *    fills or returns early in the same cases, lut2_gather.c:515-523, and its
 *    Python decoders raise ValueError, pack_codec.py:129-137).
 *  - Packed weights are the reference's own wire blobs, byte for byte,
 *    uploaded to device memory unchanged:
 *      SG8\x01 : u32 group | f32[groups][2] (min,max) | u8[numel]      (pack_codec.py:13-68)
 *      TR2\x03..\x07 : u32 group | records[groups] | 2-bit codes       (trinity_codec.py:52-58)
 *      TR2\x01 : f32 codebook[4] | 2-bit codes (one codebook per tensor)  (trinity_codec.py:612-625)
 *    The fast GEMV paths need the code payload 16-byte aligned; other
 *    placements use the general (slower) path with identical results.
 *  - All arithmetic is fp32.  Dequantised weights are bit-identical to the
 *    reference decoders; GEMV results differ from the reference C only by
 *    reduction order.
 *  - No entry point falls back to the CPU.
 */
#ifndef RWKV_B200_H
#define RWKV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RWKVB_ABI_VERSION 1

#define RWKVB_OK 0
#define RWKVB_EARG 1        /* invalid arguments / malformed blob */
#define RWKVB_EALLOC 2      /* device allocation failed */
#define RWKVB_ECUDA 3       /* a CUDA runtime call failed */
#define RWKVB_ETIMEOUT 4    /* a bounded device wait gave up */
#define RWKVB_EUNSUPPORTED 5
#define RWKVB_ESCRATCH 6     /* request larger than a fixed static scratch buffer */

/* blob kinds: the 4th magic byte ("SG8\x01" is kind 1, "TR2\xNN" is kind NN) */
#define RWKVB_KIND_SG8 1u
#define RWKVB_KIND_LUT2_F32 3u     /* TR2\x03: fp32 centroids, 16-byte records */
#define RWKVB_KIND_LUT2_F16 4u     /* TR2\x04: fp16 centroids, 8-byte records */
#define RWKVB_KIND_LUT2_RES 5u     /* TR2\x05: fp16 centroids + 2 residuals, 16-byte records */
#define RWKVB_KIND_LUT2_IN_F16 6u  /* TR2\x06: as \x04, tensor stored input-major */
#define RWKVB_KIND_LUT2_IN_RES 7u  /* TR2\x07: as \x05, tensor stored input-major */
/* TR2\x01, the legacy per-tensor LUT2 (trinity_codec.py:51, :612-625): one fp32
 * codebook of 4 values at byte 4, then the 2-bit codes of the flattened tensor
 * (LSB first) at byte 20.  Its fourth magic byte equals SG8's, hence its own id. */
#define RWKVB_KIND_LUT2_TENSOR 33u

/* One packed matrix of checkpoint shape [rows, cols] resident in device memory. */
typedef struct rwkvb_packed {
  const uint8_t* data; /* device pointer to the blob's first byte (the magic) */
  uint64_t bytes;      /* blob length */
  uint32_t kind;       /* RWKVB_KIND_* */
  uint32_t group_size; /* elements per group */
  int32_t rows;
  int32_t cols;
} rwkvb_packed;

/* Bytes of one per-group record (the codebook for RWKVB_KIND_LUT2_TENSOR). */
static inline uint32_t rwkvb_lut2_record_bytes(uint32_t kind) {
  return (kind == RWKVB_KIND_LUT2_F16 || kind == RWKVB_KIND_LUT2_IN_F16) ? 8u : 16u;
}

/* Library ABI version (RWKVB_ABI_VERSION). */
int rwkvb_version(void);

/* Human-readable text for a status code (static storage). */
const char* rwkvb_status_string(int status);

/* Parse and validate a blob header and fill `out`.
 * `header` = host copy of at least the first 8 blob bytes.  Validation follows
 * decode_scale_u8_grouped_to_tensor (pack_codec.py:126-137: magic, group > 0,
 * exact length 8 + groups*8 + numel) and decode_trinity_lut2_to_tensor
 * (trinity_codec.py:769-790: grouped kinds 3..7, group > 0, records + codes fit). */
int rwkvb_packed_init(rwkvb_packed* out, const uint8_t* header, uint64_t blob_bytes,
                      const uint8_t* device_blob, int32_t rows, int32_t cols);

/* out[rows*cols] = decoded weights in checkpoint order, fp32, bit-exact.
 * Replaces decode_scale_u8_grouped_to_tensor (pack_codec.py:126-144) and the
 * grouped branch of decode_trinity_lut2_to_tensor (trinity_codec.py:769-885). */
int rwkvb_dequant_f32(float* out, const rwkvb_packed* w, void* stream);

/* y[rows] = W @ x[cols].  SG8 replaces scale_u8_grouped_gemv_f32_export
 * (lut2_gather.c:491-496); LUT2 kinds replace trinity_grouped_lut2_gemv_f32_export
 * (lut2_gather.c:328-333); the per-tensor LUT2 replaces lut2_gemv_f32_export
 * (lut2_gather.c:179-211, :253-262), including its row walk (row r reads the
 * codes from byte (r*cols)/4 on, low bits first, which differs from the
 * flattened order when cols % 4 != 0); the dispatch mirrors lut2_gemv
 * (lut_gemm_fused.py:1095-1192). */
int rwkvb_gemv_f32(float* y, const rwkvb_packed* w, const float* x, void* stream);

/* n_mats (1..4) GEMVs with distinct inputs in one launch: y_out[m][rows] =
 * W_m @ x_m, every W_m of one shape [rows, cols] and any supported kind
 * (HOST arrays of descriptors / device input pointers).  Replaces the four-
 * and three-map batches scale_u8_grouped_tmix_gemv_f32_export (lut2_gather.c:
 * 1427-1437) and lut2_tmix_gemv_f32_export / lut2_tmix_qkv_gemv_f32_export
 * (lut2_gather.c:1517-1595, flattened code order), behind
 * lut2_tmix_gemv_batched (lut_gemm_fused.py:1724-1769). */
int rwkvb_tmix_gemv_f32(float* y_out, const rwkvb_packed* const* w, const float* const* x, int32_t n_mats,
                        void* stream);

/* Opt-in activation-INT8 SG8 GEMV: per input group of the weight's group size,
 * x is quantised to int8 with scale max|x| / 127 (1 when max|x| <= 1e-12),
 * rounding half away from zero, clamped to +-127; the exact fp32 sum of the
 * group is kept for the minimum term:
 *   y[row] = sum_g min_g * sum(x_g) + (max_g - min_g) / 255 * scale_g * sum(q * x_i8)
 * with an exact integer dot.  Changes rounding against the float path, like
 * the reference, which keeps it behind RWKV_LUT_ACTIVATION_INT8.  cols not a
 * multiple of the group: the float GEMV (as the reference falls back).  The
 * int8 activations live in a stream-ordered allocation made by the call.
 * Replaces scale_u8_grouped_i8_gemv_f32_export (lut2_gather.c:612-796). */
int rwkvb_gemv_sg8_i8_f32(float* y, const rwkvb_packed* w, const float* x, void* stream);

/* The activation-INT8 form of rwkvb_tmix_qkv_gemv_f32 (three SG8 maps of one
 * group size, each input quantised on its own).  Replaces
 * scale_u8_grouped_tmix_qkv_i8_gemv_f32_export (lut2_gather.c:1451-1515). */
int rwkvb_tmix_qkv_i8_gemv_f32(float* y_out, const rwkvb_packed* const* w3, const float* const* x3, void* stream);

/* y[cols] = x[rows] @ W for a row-major SG8 W (compact TMix adapters).
 * Replaces scale_u8_grouped_transposed_gemv_f32_export (lut2_gather.c:939-944). */
int rwkvb_transposed_gemv_f32(float* y, const rwkvb_packed* w, const float* x, void* stream);

/* y_out[3][n] = (Wr @ xr, Wk @ xk, Wv @ xv) in one launch; `w3` and `x3` are HOST
 * arrays of 3 descriptors / device pointers, all W of one shape [n, m].
 * Replaces scale_u8_grouped_tmix_qkv_gemv_f32_export (lut2_gather.c:1436-1449)
 * behind lut2_tmix_qkv_gemv_batched (lut_gemm_fused.py:1771-1817). */
int rwkvb_tmix_qkv_gemv_f32(float* y_out, const rwkvb_packed* const* w3,
                            const float* const* x3, void* stream);

/* Fused RWKV-7 TMix adapters (all SG8):
 *   w = W2 @ tanh(W1 @ xw); a = sigmoid(a0 + A2 @ (A1 @ xa));
 *   g = G2 @ sigmoid(G1 @ xg); v = V2 @ (V1 @ xv)   (x @ W convention)
 * `mats` = HOST array of 8 descriptors w1,w2,a1,a2,g1,g2,v1,v2 (the v pair is
 * ignored when has_v == 0); `xs` = HOST array of 4 device pointers xw,xa,xg,xv.
 * Replaces scale_u8_grouped_transposed_tmix_fused_f32_export (lut2_gather.c:1006-1103). */
int rwkvb_tmix_adapters_f32(float* w_out, float* a_out, float* g_out, float* v_out,
                            const rwkvb_packed* const* mats, const float* const* xs,
                            const float* a0, int has_v, void* stream);

/* y = Wv @ relu(Wk @ x)^2 (RWKV-7 channel mix).  The ffn-wide intermediate lives
 * in a stream-ordered device allocation made by this call.
 * Replaces scale_u8_grouped_cmix_gemv_f32_export (lut2_gather.c:505-610). */
int rwkvb_cmix_gemv_f32(float* y, const rwkvb_packed* key, const rwkvb_packed* value,
                        const float* x, void* stream);

/* Same result as rwkvb_cmix_gemv_f32, without any device allocation: the
 * ffn-wide intermediate lives in a file-scope static device buffer of
 * RWKVB_CMIX_NOALLOC_MAX_FFN floats (64 KiB) per device.
 *   - key->rows (the ffn width) above RWKVB_CMIX_NOALLOC_MAX_FFN returns
 *     RWKVB_ESCRATCH before touching the device.
 *   - The first call on a device (with that device current) resolves the
 *     buffer's address with cudaGetSymbolAddress; make that first call before
 *     any stream capture.  The address is kept per context: after a
 *     cudaDeviceReset the next call resolves it again in the new context.
 *     No call makes an allocating CUDA call.
 *   - Nothing has to start at zero: the key GEMV writes every intermediate
 *     element before the value GEMV reads it.
 *   - One buffer per device: calls that overlap on one device (different
 *     streams, or threads without ordering) race on it.  Serialise them.
 * For callers that must not allocate device memory per call: a decode loop
 * whose HBM is fully committed to resident weight arenas (a per-call
 * allocation can fail mid-generation), and processes on devices or drivers
 * without stream-ordered memory pools.
 * No counterpart in the reference (its C kernel mallocs the intermediate on
 * every call, lut2_gather.c:542-568). */
#define RWKVB_CMIX_NOALLOC_MAX_FFN 16384
int rwkvb_cmix_gemv_f32_noalloc(float* y, const rwkvb_packed* key, const rwkvb_packed* value,
                                const float* x, void* stream);

/* Batched SG8 product on the tcgen05 tensor cores:
 *   y[b][n] = sum_k W[n][k] x[b][k],   x [batch][cols] fp32, y [batch][rows] fp32
 * for 1 <= batch <= 64.  W: SG8 with group 64 or 128, rows and cols multiples
 * of 128, code payload 16-byte aligned (else RWKVB_EUNSUPPORTED).  Integer MMA
 * on the raw codes and a 3-digit split of x (error <= 6.2e-8 of each group's
 * largest |x|), per-group fp32 scaling, deterministic split-K reduction.
 * `err_word` (device int, may be NULL) gets RWKVB_ETIMEOUT's flag bit if a
 * bounded device wait gave up.  The tensor maps and the device workspace of a
 * (weight, batch) pair are built on its first call and kept (up to 32 pairs per
 * process); calls with the same weight and batch on different streams at the
 * same time share that workspace and must be serialised by the caller.  Replaces the batched (2-D x) branch of
 * lut2_linear_forward (rwkv_ssd/runtime/lut_gemm_fused.py:1820-1851), which
 * decodes W and calls torch.nn.functional.linear. */
int rwkvb_gemm_sg8_f32(float* y, const rwkvb_packed* w, const float* x, int32_t batch,
                       int32_t* err_word, void* stream);

/* WKV7 recurrent state update for `batch` x `n_head` heads of size N = head_size (64):
 *   d = decay(w);  S = S * diag(d) + (S @ -kk) (kk*a)^T + v k^T;  y = S @ r
 * state [batch][n_head][N][N] fp32 (value index major), vectors [batch][n_head*N].
 * decay_mode 0: d = exp(-0.606531 * sigmoid(w))   (rwkv7_linear.py:314, the model form)
 * decay_mode 1: d = exp(-exp(w))                 (the kernel microbenchmark form)
 * Replaces the state-update block of tmix_one_fused (rwkv7_linear.py:314-337). */
int rwkvb_wkv7_f32(float* state, float* y, const float* r, const float* w, const float* k,
                   const float* v, const float* kk, const float* a, int batch, int n_head,
                   int head_size, int decay_mode, void* stream);

/* ------------------------------------------------------------------------------
 * Decode engine: the whole packed RWKV-7 token step on the device.
 * Replaces, per token, forward_block_packed (packed_block_forward.py:76-166) for
 * every layer, the embedding + ln0 (rwkv7_skeleton.py:74-81), ln_out + packed head
 * (rwkv7_forward.py:791-809) and greedy argmax (sampling.py:161-163).
 * ------------------------------------------------------------------------------ */

/* Per-layer tensors.  Matrices are packed descriptors; vectors are fp32 [n_embd]
 * device arrays (r_k flattened [n_head*head_size], already decoded). */
typedef struct rwkvb_layer_desc {
  rwkvb_packed att_r, att_k, att_v, att_o;
  rwkvb_packed w1, w2, a1, a2, g1, g2, v1, v2; /* v1/v2 unused on layer 0 */
  rwkvb_packed ffn_key, ffn_value;
  const float *ln1_w, *ln1_b, *ln2_w, *ln2_b;
  const float *x_r, *x_w, *x_k, *x_v, *x_a, *x_g;
  const float *w0, *a0, *v0, *k_k, *k_a, *r_k;
  const float *lnx_w, *lnx_b, *ffn_x_k;
} rwkvb_layer_desc;

typedef struct rwkvb_model_desc {
  int32_t n_layer, n_embd, head_size, ffn, vocab;
  rwkvb_packed emb;  /* [vocab, n_embd] */
  rwkvb_packed head; /* [vocab, n_embd] */
  const float *ln0_w, *ln0_b, *ln_out_w, *ln_out_b;
  const rwkvb_layer_desc* layers; /* HOST array of n_layer descriptors */
} rwkvb_model_desc;

typedef struct rwkvb_engine rwkvb_engine;

/* Creates an engine on the current device.  The engine copies the descriptors,
 * owns the recurrent state, activations and scratch, and borrows the weights
 * (they must stay resident while the engine lives).
 * flags: bit0 = no CUDA-graph capture of the multi-kernel token step;
 *        bit1 = no programmatic dependent launch between phase kernels;
 *        bit2 = no persistent kernel (always use the multi-kernel step);
 *        bit3 = record persistent-kernel phase timestamps (rwkvb_engine_trace);
 *        bit8 = bits 4..7 give an explicit L2-prefetch distance in phases;
 *        bit9 = load the persistent kernel's weight stream without the L2
 *               evict-first policy (default: weights evict first, so the
 *               state and activations re-read every layer stay in L2);
 *        bits 12..15 = ring slots of weight tiles in flight per SM in the
 *               persistent kernel, 3..8 (0: the default, 3 -- deeper rings
 *               delay the kernel's own small loads behind the weight stream);
 *        bit16 = persistent kernel: FFN value-projection units in row order
 *               with fp32 accumulation (default: column-chunk order, so each
 *               SM builds the activation digits of only its one or two chunks,
 *               and 2^-32 fixed-point accumulation). 
 * When every projection is SG8 with one power-of-two group size and the
 * 16-byte layout that rwkvb upload placement gives, decode runs as ONE
 * cooperative persistent launch per call (all tokens, all layers); otherwise
 * (LUT2, irregular shapes) each token step is a CUDA graph of phase kernels. */
int rwkvb_engine_create(const rwkvb_model_desc* desc, uint32_t flags, rwkvb_engine** out);
int rwkvb_engine_destroy(rwkvb_engine* e);

/* Residency tiers: an engine whose streamed layers live in pinned host memory
 * and are staged into a ring of device slots on every token step, for models
 * larger than the HBM budget given to them.  Replaces the reference's staging
 * ring and prefetch planner (rwkv_ssd/runtime/staging.py:40-129,
 * prefetch.py:1-131) and its resident / streamed split (residency.py:1-118).
 * `desc` describes every layer; a streamed layer's matrices point into the
 * device slot slot_of_layer[i] (>= 0; -1: resident layer), at the offsets of
 * its image host_src[i] (layer_bytes of PINNED host memory, the layer's blobs
 * laid out as in the slot).  Per step, on a copy stream forked from the step's
 * stream: the H2D copy of each streamed layer's image into its slot, after the
 * kernels of the slot's previous user in the step; the layer's kernels wait
 * for their copy.  With n_slots slots the copies run up to n_slots streamed
 * layers ahead of the compute (2: one layer of lookahead).  The step is the
 * multi-kernel step (and its CUDA graph, copies included).  The engine borrows
 * the host images and the slots. */
typedef struct rwkvb_stage_desc {
  int32_t n_slots;
  const int32_t* slot_of_layer;  /* HOST [n_layer] */
  const void* const* host_src;   /* HOST [n_layer]; NULL for resident layers */
  void* const* slot_dev;         /* HOST [n_slots] device pointers */
  uint64_t layer_bytes;
} rwkvb_stage_desc;
int rwkvb_engine_create_staged(const rwkvb_model_desc* desc, const rwkvb_stage_desc* stage, uint32_t flags,
                               rwkvb_engine** out);

/* Device pointers of the recurrent state, laid out as RecurrentState.rwkv7_state
 * (state_cache.py:38-56, rwkv7_skeleton.py:121-131): per layer l
 *   att_x + l*n_embd              x_prev of the time mix   [n_embd]
 *   wkv   + l*n_head*N*N          WKV7 state               [n_head][N][N]
 *   ffn_x + l*n_embd              x_prev of the channel mix [n_embd]
 * `logits` = the last step's fp32 logits [vocab]. */
int rwkvb_engine_buffers(rwkvb_engine* e, float** att_x, float** wkv, float** ffn_x,
                         float** logits);

/* Zero the recurrent state (rwkv7_skeleton.py:121-131). */
int rwkvb_engine_reset(rwkvb_engine* e, void* stream);

/* Run one token step per entry of `tokens` (HOST array), in order, updating the
 * state; logits of the last step stay in the engine's logits buffer. */
int rwkvb_engine_forward(rwkvb_engine* e, const int32_t* tokens, int32_t n_tokens, void* stream);

/* Greedy decode: step 0 consumes `first_token`; step i>0 consumes step i-1's
 * argmax, all on the device.  Writes the n argmax ids to out_tokens (HOST).
 * Synchronises `stream` before returning. */
int rwkvb_engine_decode_greedy(rwkvb_engine* e, int32_t first_token, int32_t n_tokens,
                               int32_t* out_tokens, void* stream);

/* Same as rwkvb_engine_decode_greedy but leaves the ids in device memory
 * (`out_tokens_dev`, n_tokens int32) and does not synchronise. */
int rwkvb_engine_decode_greedy_async(rwkvb_engine* e, int32_t first_token, int32_t n_tokens,
                                     int32_t* out_tokens_dev, void* stream);

/* Streamed greedy decode for callers that consume tokens as they are made
 * (the token callback, cancellation and deadline of the reference's
 * decode_greedy, pack_backend.py:71-84 and generation_control.py:19-35): the
 * whole generation is ONE persistent launch, and the host learns of each token
 * through mapped pinned host memory instead of a launch and a synchronisation
 * per token.
 *
 * rwkvb_engine_host_ring: the engine's ring (allocated at the first call):
 *   ids[cap]  each step's greedy id: rwkvb_engine_decode_stream sets ids[0..n)
 *             to -1 and the device replaces slot i with step i's id (one 32-bit
 *             store) as soon as the step ends, so a reader polls the slot it
 *             waits for;
 *   *count    ids written so far (exact once the launch has ended);
 *   *cancel   read by the device once per token and acted on at the following
 *             token: non-zero stops the decode at a token boundary.
 * rwkvb_engine_decode_stream: greedy decode of n <= cap steps from first_token
 * (step 0 consumes it, step i > 0 consumes step i-1's id), streamed into the
 * ring; resets ids[0..n), *count and *cancel, launches and returns without
 * synchronising.  No step waits on the host or the bus.
 * The previous streamed decode of the engine must have finished (its stream
 * synchronised) before the next call.  When cancelled, *count gives the steps
 * that ran; the state is that after those steps.  out_tokens_dev (device, may be
 * NULL) receives the n ids as well (valid up to *count).  Persistent engines
 * only (RWKVB_EUNSUPPORTED otherwise).
 * rwkvb_engine_check: synchronise `stream` and report (then clear) a device
 * error of the engine's launches (RWKVB_ETIMEOUT, RWKVB_EARG for a bad token). */
int rwkvb_engine_host_ring(rwkvb_engine* e, int32_t** ids, volatile uint32_t** count, volatile int32_t** cancel,
                           int32_t* cap);
int rwkvb_engine_decode_stream(rwkvb_engine* e, int32_t first_token, int32_t n_tokens, int32_t* out_tokens_dev,
                               void* stream);
int rwkvb_engine_check(rwkvb_engine* e, void* stream);

/* Timestamps (ns, %globaltimer) of the last persistent launch, recorded when
 * the engine was created with flag bit 3; copies min(cap, 262144) values to
 * host `out`:
 *   [0, 131072): phase marks, [2][65536] (first CTA, last CTA): per token the
 *     token start, per layer 16 marks (A start, A prep (ln1, shift state, r/k/v
 *     digits), A units, A items, B barrier, B done, C barrier, C prep, C units,
 *     D barrier, D prep (loads, ln2, digits), D units, E barrier, E slices,
 *     E prep, E units), then head barrier, head prep, head units;
 *   [131072, 262144): ring events of the first CTA, 3 per stage s (s < 43690):
 *     producer issue, consumer wait end, consumer release.
 * The GPU counterpart of the reference's per-layer LayerTiming rows
 * (runtime/metrics.py:26-58). */
int rwkvb_engine_trace(rwkvb_engine* e, uint64_t* out, int32_t cap, int32_t* n_out);

/* Kernel launches per token step (for launch accounting). */
int rwkvb_engine_launches_per_step(rwkvb_engine* e, int32_t* out);

/* ------------------------------------------------------------------------------
 * Batched decode: `batch` (1..64) independent sessions of one model advance one
 * token per step together, every projection (r/k/v/o, FFN key/value, head) a
 * tcgen05 batched GEMM (as rwkvb_gemm_sg8_f32), the adapters, WKV7, LayerNorms
 * and argmax in small kernels; one step is a CUDA graph.  Per session the step
 * is forward_block_packed for every layer + head + greedy argmax, as the
 * reference runs it session by session (its batched path, rwkv7_batch, lives in
 * the un-vendored ChatRWKV package).
 * Requirements: every r/k/v/o/FFN/head matrix SG8 with one group size (64 or
 * 128), or every one TR2\x04 (LUT2, fp16 codebooks) with group 64; n_embd, ffn
 * and vocab multiples of 128; adapters and embedding any codec.  SG8 products
 * are integer tcgen05 GEMMs over digit rows; LUT2 products decode the 2-bit
 * codes to fp16 tiles in shared memory for fp16 tcgen05 GEMMs (activations as
 * two fp16 planes, fp32 accumulation).  LUT2 engines run prefill positions as
 * decode steps; tensor parallelism needs SG8.
 * ------------------------------------------------------------------------------ */
typedef struct rwkvb_batch rwkvb_batch;

/* flags: bit0 = run the step as plain launches (no CUDA graph);
 *        bit1 = no programmatic dependent launch between the step's kernels
 *               (default: each kernel may start while the previous one
 *               finishes; the GEMMs stream their first weight tiles before
 *               waiting on it).  Always off under tensor parallelism;
 *        bit2 = LUT2 engines: products on the CUDA cores (fp32 FMA) instead
 *               of the tensor cores (a cross-check path);
 *        bits 16..19 = tensor parallelism with peer exchange: wall-time limit
 *               of one exchange wait in units of 100 ms (0: 5 s).  When a
 *               peer does not arrive in time the step's later exchanges return
 *               at once and the next synchronising call reports RWKVB_ETIMEOUT
 *               (clearing the error word). */
int rwkvb_batch_create(const rwkvb_model_desc* desc, int32_t batch, uint32_t flags, rwkvb_batch** out);

/* Tensor parallelism across the GPUs of one node (one process per GPU), the
 * head-sharded split for models such as the 7.2B one: each rank holds the attention heads
 * of its shard (r/k/v rows, the matching columns of the adapter second stages
 * and of the output projection, the heads' per-channel vectors), a slice of the
 * FFN (key rows, the matching value columns) and a slice of the vocabulary
 * (head rows); embedding, LayerNorms, token-shift mixes and adapter first stages
 * are replicated.  Per layer the output and value projections yield partial
 * sums that the host's `collective` callback all-reduces (kind 0: sum of fp32 in
 * place, send == recv); the per-session argmax bests (float value, int32 index
 * bits, 8 bytes per session) are all-gathered (kind 1: `bytes` from every rank
 * into recv in rank order).  The callback is called on the engine's stream
 * while the step is recorded (it is captured into the step's CUDA graph when
 * the collective library supports capture) and must issue the collective on
 * that stream's order.  `local` describes this rank's shard: att r/k/v
 * [Ca][n_embd], att_o [n_embd][Ca], w2/a2/g2/v2 [rank][Ca], ffn_key [ffn][n_embd],
 * ffn_value [n_embd][ffn], head [vocab_local][n_embd]; n_embd the full width,
 * vocab the full embedding vocabulary. */
typedef void (*rwkvb_collective_fn)(int32_t kind, void* send, void* recv, int64_t bytes, void* stream, void* user);
typedef struct rwkvb_tp_desc {
  int32_t rank, size;        /* this rank, ranks (>= 2) */
  int32_t vocab_offset;      /* first vocabulary row of this rank's head shard */
  rwkvb_collective_fn collective;
  void* user;
  /* Optional (all ranks or none; size <= 8): peer[r] = rank r's exchange buffer
   * (rwkvb_ipc_alloc on rank r, rwkvb_ipc_open elsewhere; peer[rank] is this
   * rank's own), rwkvb_batch_tp_exchange_bytes bytes each.  When set, the
   * all-reduces and the argmax gather run in the engine's own kernels over
   * NVLink -- plain peer loads and stores, epoch flags with bounded waits
   * (RWKVB_ETIMEOUT from the next synchronising call when a peer does not
   * arrive), every rank summing in rank order -- and `collective` is unused. */
  void* const* peer;
} rwkvb_tp_desc;
int rwkvb_batch_create_tp(const rwkvb_model_desc* local, int32_t batch, const rwkvb_tp_desc* tp, uint32_t flags,
                          rwkvb_batch** out);
/* Bytes of one rank's exchange buffer for rwkvb_tp_desc.peer. */
int rwkvb_batch_tp_exchange_bytes(const rwkvb_model_desc* local, int32_t batch, uint64_t* bytes);
/* Device memory other processes of this node can map (CUDA IPC), zeroed:
 * `handle` receives 64 opaque bytes to pass to them. */
int rwkvb_ipc_alloc(uint64_t bytes, void** dev_ptr, uint8_t* handle);
int rwkvb_ipc_free(void* dev_ptr);
/* Map another process's rwkvb_ipc_alloc buffer into this one (current device). */
int rwkvb_ipc_open(const uint8_t* handle, void** dev_ptr);
int rwkvb_ipc_close(void* dev_ptr);
/* Record the token step as a CUDA graph now (once; a no-op without graphs),
 * instead of at the first step.  Nothing runs.  Under tensor parallelism every
 * rank calls it and the ranks agree that all captures succeeded before any
 * rank launches a step: a graph holding collectives must never run on some
 * ranks only. */
int rwkvb_batch_prepare(rwkvb_batch* e, void* stream);
int rwkvb_batch_destroy(rwkvb_batch* e);

/* Device state, per layer l and session b (each block as in rwkvb_engine_buffers):
 *   att_x + (l*batch + b)*n_embd,  wkv + (l*batch + b)*n_head*N*N,  ffn_x + (l*batch + b)*n_embd;
 * logits [batch][vocab] of the last step.  Under tensor parallelism n_head is
 * this rank's heads (Ca / 64) and logits hold this rank's vocabulary rows
 * [vocab_offset, vocab_offset + vocab_local). */
int rwkvb_batch_buffers(rwkvb_batch* e, float** att_x, float** wkv, float** ffn_x, float** logits);
int rwkvb_batch_reset(rwkvb_batch* e, void* stream);

/* One step: session b consumes tokens[b] (HOST array of `batch` ids). */
int rwkvb_batch_forward(rwkvb_batch* e, const int32_t* tokens, void* stream);

/* Sequence prefill: session b consumes tokens[b*n .. b*n+n) (HOST, row-major
 * [batch][n]) in order, with the result of n rwkvb_batch_forward steps.
 * Positions run in chunks of P = 64 / batch: every projection of a chunk is ONE
 * tcgen05 GEMM over batch * P rows (session, position); the token shift and
 * WKV7 follow positions in order inside the chunk (state in registers); the
 * head runs once, for the last position.  Positions past the last full chunk
 * (and every position when P < 2) run as single steps.  Replaces the prompt
 * loop of the reference's sequence prefill (rwkv7_forward.py:1046-1175,
 * rwkv7_batch.py:94-220) for packed models. */
int rwkvb_batch_prefill(rwkvb_batch* e, const int32_t* tokens, int32_t n, void* stream);

/* n greedy steps; step 0 consumes the argmax of the current logits of every
 * session, step i > 0 the argmax of step i-1.  ids [n][batch] to HOST memory
 * (synchronises) or device memory (_async, does not synchronise). */
int rwkvb_batch_decode_greedy(rwkvb_batch* e, int32_t n, int32_t* out_tokens, void* stream);
int rwkvb_batch_decode_greedy_async(rwkvb_batch* e, int32_t n, int32_t* out_tokens_dev, void* stream);

/* Kernel launches per batched step. */
int rwkvb_batch_launches_per_step(rwkvb_batch* e, int32_t* out);

#ifdef __cplusplus
}
#endif

#endif /* RWKV_B200_H */
