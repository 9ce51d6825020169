/* C ABI of libowsmdec.so: the OWSM Transformer decoder call (embedding -> L pre-LN layers of masked
 * self-attention over a per-row KV cache, cross-attention over precomputed encoder K/V and a ReLU FFN ->
 * final LayerNorm -> vocabulary projection -> argmax, or log-softmax + top-K with a KV-cache reorder)
 * as one persistent CUDA kernel for sm_100a (B200).
 *
 * Plain C types only: device pointers as void*, sizes as int / int64_t, the CUDA stream as void*.
 * Every function returns OWSM_DEC_OK (0) or a negative error code; no exception crosses the ABI.
 *
 * Correspondence with owsm-trt (the Python interface this library replaces):
 *   owsm_dec_create      <- MegaDecoder.__init__        src/owsm_trt/megakernel.py:548-614
 *                           (LayerNorm folding :564-570, per-layer weight stacks :577-599)
 *   owsm_dec_plan        <- MegaDecoder.step_fn scratch src/owsm_trt/megakernel.py:624-650,
 *                           RingDecoder.step_fn         src/owsm_trt/megakernel_ring.py:794-830
 *   owsm_dec_step        <- the returned run()          src/owsm_trt/megakernel.py:667-672,
 *                           megakernel_ring.py:852-853 (pred / notime: :794-799)
 *   owsm_dec_step_verify <- run() + kernels.choose + kernels.accept  src/owsm_trt/runtime.py:1292-1316
 *   owsm_dec_beam_step   <- run() followed by BeamSession._select step 1 and the cache reorder
 *                           src/owsm_trt/runtime.py:1399-1413
 *   owsm_dec_get_error   <- MegaDecoder.check           src/owsm_trt/megakernel.py:616-622
 */
#ifndef OWSM_DEC_H
#define OWSM_DEC_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OWSM_DEC_OK 0
#define OWSM_DEC_ERR_ARG (-1)      /* invalid argument (shape, pointer, alignment) */
#define OWSM_DEC_ERR_CUDA (-2)     /* a CUDA runtime call failed */
#define OWSM_DEC_ERR_TIMEOUT (-3)  /* a bounded in-kernel wait gave up (results of that call are garbage) */
#define OWSM_DEC_ERR_LIMIT (-4)    /* the call exceeds a supported maximum (rows x window, head size, ...) */

#define OWSM_DEC_F32 0 /* weight element type given to owsm_dec_create */
#define OWSM_DEC_F16 1

/* Model shapes (OWSMConfig dec_layers, d_model, dec_heads, dec_ffn, vocab_size; src/owsm_trt/config.py:15-30). */
typedef struct OwsmDecDims {
  int L, D, H, F, V;
  int max_pos;  /* rows of the positional table */
  float eps;    /* LayerNorm eps (1e-12, src/owsm_trt/modeling.py:25) */
  float xscale; /* embedding scale sqrt(D) (modeling.py:481) */
} OwsmDecDims;

/* One layer's parameters, device pointers, row-major [out, in] as torch.nn.Linear stores them
 * (element type = weight_dtype; vectors always fp32). wq/wk/wv are the self-attention projections
 * (DecoderLayer.self_attn, modeling.py:461-469); if wk == NULL, wq is the fused [3D, D] matrix
 * (MultiHeadedAttention.fuse_qkv, modeling.py:153-161) and bq the fused bias. */
typedef struct OwsmDecLayer {
  const void *wq, *wk, *wv;
  const float *bq, *bk, *bv;
  const void* wo;
  const float* bo;
  const void* wcq; /* src_attn.linear_q */
  const float* bcq;
  const void* wco; /* src_attn.linear_out */
  const float* bco;
  const void* w1; /* feed_forward.w_1 [F, D] */
  const float* b1;
  const void* w2; /* feed_forward.w_2 [D, F] */
  const float* b2;
  const float *ln1_g, *ln1_b, *ln2_g, *ln2_b, *ln3_g, *ln3_b;
} OwsmDecLayer;

typedef struct OwsmDecWeights {
  int weight_dtype;         /* OWSM_DEC_F32 or OWSM_DEC_F16 */
  const void* emb;          /* [V, D] */
  const float* pe;          /* [max_pos, D] positional table (fp32) */
  const OwsmDecLayer* layers; /* host array of L */
  const float *lnf_g, *lnf_b; /* after_norm */
  const void* wout;         /* output_layer [V, D] */
  const float* bout;
} OwsmDecWeights;

typedef struct OwsmDec OwsmDec;         /* packed weights on one device */
typedef struct OwsmDecPlan OwsmDecPlan; /* scratch + schedule for one call shape */

/* Pack the weights (LayerNorms folded into the following GEMMs, fp16, tensor-core fragment order) on
 * `device`. The given buffers may be freed afterwards. `programs` = CTAs of the persistent kernel
 * (0: one per SM). */
int owsm_dec_create(const OwsmDecDims* dims, const OwsmDecWeights* w, int device, int programs, OwsmDec** out);
void owsm_dec_destroy(OwsmDec* h);

/* Shapes of a call: R rows x S new tokens, self-KV cache capacity C, T encoder frames; cross K/V hold
 * R / rows_per_utt utterances (rows_per_utt = 1: one per row, owsm-trt's layout; = beam: the beam
 * hypotheses of an utterance read its K/V once). beam > 0 prepares owsm_dec_beam_step with that beam
 * (R = batch * beam, utterance-major). Allocates the call's scratch on the handle's device. */
int owsm_dec_plan(OwsmDec* h, int R, int S, int C, int T, int rows_per_utt, int beam, OwsmDecPlan** out);
void owsm_dec_plan_destroy(OwsmDecPlan* p);

/* One decoder call on `stream` (cudaStream_t; NULL = legacy default). Device pointers:
 *   tokens  int64 [R, S], row stride tok_stride (elements)      offset int64 [R], stride off_stride
 *   self_k, self_v fp16 [L, R, H, C, dk]: read at slots < offset[r], written at offset[r] .. +S-1
 *   cross_k, cross_v fp16 [L, R / rows_per_utt, H, T, dk]
 *   enc_len int32 [R / rows_per_utt] or NULL: frames of each utterance (key-padding mask), clamped to [1, T]
 *   logits fp32 [R, S, V] (written)    new_kv fp16 [L, 2, R, H, S, dk] (written)
 *   pred int64 [R, S] or NULL: argmax of the logits (first index on ties)
 *   notime uint8 [R] or NULL: rows whose argmax leaves out ids first_time..last_time
 * No host synchronisation; capturable in a CUDA graph (all pointers are fixed in the graph). */
int owsm_dec_step(OwsmDecPlan* p, void* stream, const int64_t* tokens, int64_t tok_stride, const int64_t* offset,
                  int64_t off_stride, void* self_k, void* self_v, const void* cross_k, const void* cross_v,
                  const int32_t* enc_len, float* logits, void* new_kv, int64_t* pred, const uint8_t* notime,
                  int first_time, int last_time);

/* A verify call of the speculative greedy session (_Bound.body, src/owsm_trt/runtime.py:1292-1316) in one launch:
 * the decoder call on the rows of `inp` -- int64 [R][inp_stride >= S + 4] = [S tokens | offset | timestamps so far |
 * last timestamp | first generated position] (runtime.py:1240-1241) -- then, in the vocabulary epilogue, the argmax
 * after every window position into pred int64 [R, S], under ESPnet's timestamp rules when rules != 0
 * (TimestampRules.forbidden + _Verify.predict, runtime.py:471-492, :1251-1267; replaces kernels.choose,
 * src/owsm_trt/kernels.py:26-66, 115-123), with notime (uint8 [R] or NULL) the rows whose primer holds
 * <notimestamps> and first_time .. last_time the timestamp ids; and, when res != NULL, per row the drafted tokens
 * accepted and the argmax after them into res int64 [R, 2] (_Verify.accept, runtime.py:1269-1278; replaces
 * kernels.accept, kernels.py:89-101, 133-136). Other arguments as owsm_dec_step; the plan is a greedy plan of
 * (R, S). */
int owsm_dec_step_verify(OwsmDecPlan* p, void* stream, const int64_t* inp, int64_t inp_stride, void* self_k,
                         void* self_v, const void* cross_k, const void* cross_v, const int32_t* enc_len,
                         float* logits, void* new_kv, int64_t* pred, const uint8_t* notime, int rules,
                         int first_time, int last_time, int eos, int64_t* res);

/* owsm_dec_step (S = 1) followed by the beam selection of BeamSession._select step 1 over the plan's
 * batch x beam rows: logp = log_softmax(logits) (fp32), cand = score[r] + logp, inactive rows LOG_ZERO,
 * top-`beam` of beam x V per utterance (ties: lower flat index) ->
 *   score fp32 [R] (overwritten with the new scores), parent int64 [R] (row each slot came from),
 *   token int64 [R]; then self_k / self_v rows are replaced by their parent's rows (slots 0 .. offset+S-1).
 * active uint8 [R].
 * shared int32 [R / beam][beam][beam] or NULL: the caller's record, per utterance, of how many leading cache
 *   slots each pair of its rows holds in common (the same keys and values). With it only the slots past that
 *   are copied from a row's parent, and the call updates the record for the next call; set every entry to the
 *   prompt length when the rows start from the same prompt (and again whenever the caches are rewritten
 *   otherwise). NULL: every slot 0 .. offset+S-1 is copied, as BeamSession's index_select does. */
int owsm_dec_beam_step(OwsmDecPlan* p, void* stream, const int64_t* tokens, int64_t tok_stride,
                       const int64_t* offset, int64_t off_stride, void* self_k, void* self_v, const void* cross_k,
                       const void* cross_v, const int32_t* enc_len, float* logits, void* new_kv, float* score,
                       const uint8_t* active, int64_t* parent, int64_t* token, int32_t* shared);

/* Read and clear the device error word of the handle's calls (synchronises the device).
 * Returns OWSM_DEC_OK, OWSM_DEC_ERR_TIMEOUT (a bounded wait gave up) or OWSM_DEC_ERR_CUDA. */
int owsm_dec_get_error(OwsmDec* h);

/* Reset a plan's inter-CTA counters after a failed call (synchronises the device). */
int owsm_dec_plan_reset(OwsmDecPlan* p);

/* Plan facts for callers and tests: programs (CTAs), ring slots, bytes of scratch. */
int owsm_dec_plan_info(const OwsmDecPlan* p, int* programs, int* ring_slots, int64_t* scratch_bytes);

/* Profiling: %globaltimer stamps of later calls of this plan into `stamps` (device, uint64
 * [stages][programs][4]: stage start, stage end, grid-barrier exit, ns spent waiting for ring slots in the stage), or NULL to
 * stop. The stage count of a call is owsm_dec_plan_stages(p, beam_call). Mirrors the megakernels' TS option
 * (src/owsm_trt/megakernel.py:421-422, :612-614). */
int owsm_dec_plan_trace(OwsmDecPlan* p, void* stamps);
/* Profiling: the event log of traced calls (128 words per CTA after the stage stamps) starts at stage
 * `first_stage` instead of the call's start. */
int owsm_dec_plan_trace_from(OwsmDecPlan* p, int first_stage);
int owsm_dec_plan_stages(const OwsmDecPlan* p, int beam_call);

/* Which kernel later plans of this handle use (no counterpart in owsm-trt, which picks its kernel by GPU):
 * 0 (default) the dense kernel (tcgen05 tensor-core GEMMs) for greedy calls of more than 32 tokens -- one launch
 * up to 64 tokens, row slices of up to 64 tokens each beyond --, the cluster kernel where the call shape allows
 * it (at most 16 tokens, or row slices of it up to 32), else the grid-stage kernel; 1 always the grid-stage
 * kernel; 2 the cluster kernel; 3 the dense kernel; with 2 and 3 owsm_dec_plan fails with OWSM_DEC_ERR_LIMIT
 * where the kernel does not apply. Existing plans keep their kernel. */
int owsm_dec_set_path(OwsmDec* h, int path);

/* The kernel a plan runs: 1 the grid-stage kernel (eight grid-wide stages per layer), 2 the cluster
 * kernel (three per layer), 3 the dense kernel (eight per layer, tcgen05 GEMMs). */
int owsm_dec_plan_kernel(const OwsmDecPlan* p);

/* Kernel launches of one call of the plan: 1, or the number of row slices a call of more than 16 tokens is cut
 * into (each slice one launch of the cluster kernel). No counterpart in owsm-trt (one launch per call). */
int owsm_dec_plan_launches(const OwsmDecPlan* p);

/* Testing hook: the in-kernel wait limit (polls) of later calls on this handle; 0 restores the default. */
int owsm_dec_set_max_spin(OwsmDec* h, uint32_t polls);

/* owsm_dec_step without a plan and without any device allocation (no counterpart in owsm-trt, whose
 * launchers allocate their scratch in step_fn). For callers that may not allocate device memory when they
 * decode: a thread that must not block on cudaMalloc (it can synchronise the device), or a host whose device
 * memory belongs to an outside pool. Greedy calls only (rows_per_utt = 1, no beam), at most 8 tokens
 * (R x S) per call and 8 MiB of scratch; a larger shape fails with OWSM_DEC_ERR_LIMIT and a message naming
 * the bytes it needs. The scratch is one fixed array of the library per device: the first call for a
 * handle and shape on a device looks it up (cudaGetSymbolAddress, with the handle's device current),
 * zeroes it and uploads the block tables, synchronously -- make that first call before any stream capture.
 * That set-up runs again, with a device-wide synchronisation, whenever the handle or any of R, S, C, T
 * differs from the previous call on the device: keep the shape fixed between calls (pad rows of finished
 * utterances instead of shrinking R) so that steady-state calls never block on the device.
 * Every call then zeroes the inter-CTA counters on `stream` and launches. Calls that overlap on one device
 * (other streams, other threads, other handles) share the array and race: run one at a time per device.
 * Arguments as owsm_dec_step, plus the call shape R, S, C (cache slots), T (encoder frames). */
int owsm_dec_step_static(OwsmDec* h, void* stream, int R, int S, int C, int T, const int64_t* tokens,
                         int64_t tok_stride, const int64_t* offset, int64_t off_stride, void* self_k, void* self_v,
                         const void* cross_k, const void* cross_v, const int32_t* enc_len, float* logits,
                         void* new_kv, int64_t* pred, const uint8_t* notime, int first_time, int last_time);

/* ---- cross-attention keys and values of the encoder output (once per utterance) ----------------------------
 * Replaces Decoder.cross_kv (src/owsm_trt/modeling.py:490-499) as TorchBackend.encode calls it after the encoder
 * (src/owsm_trt/runtime.py:63-74): for every layer, enc @ W_k^T + b_k and enc @ W_v^T + b_v, split into heads of
 * 64, as one tcgen05 GEMM over all layers (fp16 in, fp32 accumulate, fp16 out). */
typedef struct OwsmXkvLayer {
  const void *wk, *wv;   /* src_attn.linear_k / linear_v weights [D, D] (weight_dtype) */
  const float *bk, *bv;  /* their biases [D] (fp32) */
} OwsmXkvLayer;
typedef struct OwsmXkv OwsmXkv;

/* Pack the L layers' K/V projections (fp16) on `device`; D = 64 H, L x 2 x D a multiple of 256. */
int owsm_xkv_create(int L, int D, int H, int weight_dtype, const OwsmXkvLayer* layers, int device, OwsmXkv** out);
/* enc fp16 [U, T, D] (contiguous) -> cross_k, cross_v fp16 [L, U, H, t_cap, 64] (frames T .. t_cap - 1 untouched);
 * all three 128-byte aligned. Asynchronous on `stream`; no allocation, capturable in a CUDA graph. */
int owsm_xkv_run(OwsmXkv* x, void* stream, const void* enc, int U, int T, int t_cap, void* cross_k, void* cross_v);
/* Read and clear the error word of the handle's runs (synchronises): OWSM_DEC_OK or OWSM_DEC_ERR_TIMEOUT. */
int owsm_xkv_get_error(OwsmXkv* x);
void owsm_xkv_destroy(OwsmXkv* x);

/* Last CUDA / argument error message of this thread ("" if none). */
const char* owsm_dec_last_error(void);

#ifdef __cplusplus
}
#endif
#endif /* OWSM_DEC_H */
