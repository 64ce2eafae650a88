/*
 * mingproj — C-ABI of the B200 (sm_100a) kernel library for the Ming-Image
 * DiT's block-linear hot path: the seven LoRA-able projections of every
 * block (to_q, to_k, to_v, to_out.0, feed_forward.w1 / w3 / w2) and the
 * per-block adaLN modulation Linear.
 *
 * Reference interface this replaces (vpipe-ming-image, paths relative to
 * that project):
 *   - the `lin` lambda of MingDitMetal::forward, src/ming-dit.cc:1763-1771
 *       lin(x, x_elem_off, QWeight, y, y_elem_off, M, N, K, lora::Stack)
 *     = `lin_base` (src/ming-dit.cc:1721-1758) + lora::Applier::apply;
 *   - `fill_mod`, src/ming-dit.cc:2266-2273 (adaLN Linear + bias + fold);
 *   - `load_qw_` / QWeight, src/ming-dit.cc:802-831 and :446-452 (pack
 *     upload), with the pack shapes pinned by tests/ming-quant-test.cc:
 *     526-530;
 *   - `bind_loras_` / `lora_for_` / `set_lora_scale`,
 *     src/ming-dit.cc:2918-3039 (slot binding and live strengths).
 *
 * Conventions:
 *   - Plain pointers and sizes only. Device pointers are CUDA device
 *     addresses on the context's device; "host or device" arguments are
 *     copied with unified addressing and may be either.
 *   - Every call returns an mp_status. Nothing aborts or exits. On failure
 *     mp_last_error() says why.
 *   - One host thread per context. Launches are stream-ordered on the
 *     stream passed in (a cudaStream_t; NULL = the legacy default stream).
 *   - Strengths in force when a projection is enqueued are captured by
 *     value into that launch.
 */
#ifndef MINGPROJ_H
#define MINGPROJ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MP_MAX_SLOTS 8     /* src/ming-dit.h:117 kMaxLoraSlots; src/ming-model-config-stage.h:45 */
#define MP_MAX_SEGMENTS 16 /* row segments with their own strength vector */
#define MP_GROUP 64        /* quantization group along K (src/ming-quant-family.h:31-47) */

typedef enum {
  MP_OK = 0,
  MP_EINVAL = 1,   /* bad argument: shape, alignment, slot, rank */
  MP_ENOMEM = 2,   /* device allocation failed */
  MP_ECUDA = 3,    /* a CUDA runtime / driver call failed (includes "no device") */
  MP_ETIMEOUT = 4  /* a device-side bounded wait gave up (reported by mp_sync_check) */
} mp_status;

typedef enum {
  MP_QUANT_AFFINE = 0,    /* w = scale * q + bias, q unsigned (w8: 0..255, w4: 0..15) */
  MP_QUANT_SYMMETRIC = 1  /* w = scale * q, q signed 8-bit (-127..127), no bias */
} mp_quant_mode;

typedef struct mp_ctx mp_ctx;
typedef struct mp_weight mp_weight;
typedef struct mp_modset mp_modset;

/* One projection weight, torch Linear layout [n out, k in]. */
typedef struct {
  int32_t n;     /* output features */
  int32_t k;     /* input features; a multiple of 64 when packed (dense: any) */
  int32_t bits;  /* 0 = dense bf16, 8 or 4 = packed codes */
  int32_t group; /* must be MP_GROUP for packed weights */
  int32_t mode;  /* mp_quant_mode, packed weights only */
} mp_weight_desc;

/* What the context ran, counted at the launch site (the reference's
 * DitEngagement, src/ming-dit.h:55-103, restricted to this path). */
typedef struct {
  int64_t linear_calls; /* projections run */
  int64_t lora_proj;    /* of those, projections carrying >= 1 live adapter */
  int64_t gemm_w8;      /* projections whose base was packed 8-bit */
  int64_t gemm_w4;      /* ... packed 4-bit */
  int64_t gemm_dense;   /* ... dense bf16 */
  int64_t lora_down;    /* rank-space pre-GEMM launches */
  int64_t modulation;   /* batched modulation launches */
  int64_t kernels;      /* kernel launches of this library */
  double flops;         /* algorithmic FLOPs: 2MNK + sum_live 2 M r (K + N), modulation 2 M N K */
  double bytes;         /* minimal HBM bytes: weights + factors + x + y */
} mp_engagement;

/* ---- context ---------------------------------------------------------- */

/* Replaces: the per-DiT Metal state set up by MingDitMetal::load_
 * (src/ming-dit.cc:1076-1415). Binds `device`; fails with MP_ECUDA when no
 * CUDA device is usable. */
int mp_create(int device, mp_ctx** out);
int mp_destroy(mp_ctx* ctx);
/* Last failure message of this context (never NULL). */
const char* mp_last_error(const mp_ctx* ctx);
/* Name of a status code. */
const char* mp_status_string(int status);
/* Synchronizes `stream` and reports device-side failures: MP_ETIMEOUT when
 * any kernel of this context gave up a bounded wait since the last check.
 * Replaces: the commit/wait of the forward (src/ming-dit.cc:2564-2571). */
int mp_sync_check(mp_ctx* ctx, void* stream);
/* Device-side wait limit in nanoseconds (default 2e9). */
int mp_set_wait_limit(mp_ctx* ctx, uint64_t ns);
/* Failure-detection self-test (no reference counterpart): launches one CTA
 * whose mbarrier wait can never complete, bounded by `limit_ns` exactly as the
 * projection kernels bound theirs. The next mp_sync_check reports MP_ETIMEOUT
 * and clears it; the context stays usable. Nothing faults or traps. */
int mp_selftest_wait(mp_ctx* ctx, uint64_t limit_ns, void* stream);

/* ---- weights ---------------------------------------------------------- */

/* Uploads one projection weight. Replaces: load_qw_ (src/ming-dit.cc:
 * 802-831) — codes uploaded raw, scales/biases narrowed to bf16 (:816-822).
 *   packed: `data` = U32 codes [n, k*bits/32] exactly as the pack stores
 *           them (code j of a word at bits [j*bits, (j+1)*bits)), `scales`
 *           and `biases` = bf16 [n, k/64] (`biases` NULL for symmetric);
 *   dense:  `data` = bf16 [n, k]; scales/biases NULL. Any k: rows are stored
 *           at a pitch padded to 8 elements and a ragged last K tile reads
 *           zeros.
 * All pointers host or device. */
int mp_weight_upload(mp_ctx* ctx, const mp_weight_desc* desc, const void* data,
                     const uint16_t* scales, const uint16_t* biases, mp_weight** out);
int mp_weight_free(mp_ctx* ctx, mp_weight* w);
/* Reads back the stored codes bytes (or dense weight) into `dst` (host or
 * device, `bytes` long) — the bit-exact upload round trip. */
int mp_weight_read_codes(mp_ctx* ctx, const mp_weight* w, void* dst, size_t bytes);

/* ---- LoRA slots ------------------------------------------------------- */

/* Binds slot `slot` of weight `w`: a = bf16 [rank, k] with the adapter's
 * alpha/rank already folded in, b = bf16 [n, rank]; host or device.
 * Replaces: Adapter::bind per projection inside bind_loras_
 * (src/ming-dit.cc:2954-2968). A shape the caller got wrong returns
 * MP_EINVAL; the caller refuses the whole slot, as bind_loras_ does
 * (:2971-2983). Rebinding a slot replaces its factors. */
int mp_lora_bind(mp_ctx* ctx, mp_weight* w, int slot, const uint16_t* a, const uint16_t* b,
                 int rank);
int mp_lora_unbind(mp_ctx* ctx, mp_weight* w, int slot);

/* Live strength of `slot` for every projection of the context. Exactly 0
 * drops the slot from the stacked contraction: the result is then
 * bit-identical to a launch without that slot. Replaces: set_lora_scale
 * (src/ming-dit.cc:3024-3039). Default 1.0. */
int mp_set_strength(mp_ctx* ctx, int slot, float s);
int mp_get_strength(const mp_ctx* ctx, int slot, float* s);
/* Per-row-segment strengths (a batch of images with their own strength
 * vectors): `s` = float [batch][MP_MAX_SLOTS], `row_starts` = int32
 * [batch + 1] token-row boundaries of the x passed to the next launches.
 * batch = 0 returns to the per-slot strengths. No counterpart in the
 * reference, which has one strength per slot; a batch of images with their
 * own strength vectors uses it. */
int mp_set_strengths_rows(mp_ctx* ctx, const float* s, const int32_t* row_starts, int batch);

/* Rows of ONE image in the x of the launches that follow, when a launch holds
 * several images of equal length with the same strengths (a CFG pass over
 * both captions); 0 (the default) = every launch is one image, unless row
 * segments are set, whose longest segment then counts. The token tile and
 * the K splits of a projection and of its rank-space pre-GEMM (which fix the
 * fp32 summation order) are chosen from this count, so each image of such a
 * batch has the bits of its own launch. Not part of the state version: a
 * graph keeps the choices of its capture. No counterpart in the reference,
 * whose batches are per image. */
int mp_set_image_rows(mp_ctx* ctx, int rows);

/* A counter that every change of a strength (to another value), of the row
 * segments or of a LoRA binding advances. Launches captured into a CUDA graph
 * keep the strengths, segments and stacked factors of their capture: a graph
 * captured at version v is replayed only while the version is still v, and
 * captured again otherwise. A launch made while its stream is capturing adds
 * to the graph what keeps it correct on every replay (the fused LoRA
 * prologue's ready flags are cleared before it), and the context never frees
 * a buffer that grows after a capture (it is kept until mp_destroy). Warm up
 * (one uncaptured call of the same shapes) before capturing, so that no
 * buffer grows and no stacked factor is rebuilt inside the capture. No
 * counterpart in the reference, which runs each block's encoder live. */
int mp_state_version(const mp_ctx* ctx, uint64_t* version);

/* ---- projections ------------------------------------------------------ */

/* y[m, n] = x[m, k] · deq(W)^T + sum over live slots s_i · (x A_i^T) B_i^T,
 * bf16 in / bf16 out, f32 accumulation, one pass over K with the adapters
 * appended as extra K tiles. x: device bf16, 16-byte aligned, ldx a
 * multiple of 8 elements. y: device bf16, 16-byte aligned, ldy >= n and a multiple of 8.
 * Over few rows per image (K split across CTA pairs) with live slots, the
 * call forks a stream of the context's own (an event record on `stream` and
 * a wait), runs the rank-space pre-GEMM and the LoRA K tiles there beside the
 * base K splits, and joins it back into `stream` before the final reduce: the
 * call stays ordered on `stream` like every other, and a CUDA-graph capture
 * of `stream` holds the fork and the join.
 * Replaces: lin (src/ming-dit.cc:1763-1771). */
int mp_linear(mp_ctx* ctx, const mp_weight* w, const void* x, int64_t ldx, void* y, int64_t ldy,
              int m, void* stream);

/* `count` projections of the same input x (q/k/v, or w1/w3): the rank-space
 * pre-GEMM of all their live adapters runs ONCE over x, then each base
 * projection. Replaces: the three (two) consecutive lin calls on `nrm` at
 * src/ming-dit.cc:2078-2080 and :2155-2156. */
int mp_linear_shared(mp_ctx* ctx, const mp_weight* const* ws, void* const* ys,
                     const int64_t* ldys, int count, const void* x, int64_t ldx, int m,
                     void* stream);

/* The FFN gate and up projections with the SwiGLU in the epilogue, one launch:
 *   h[m, n] = bf16(g / (1 + exp(-g)) * u),  g = bf16(lin(x, w1)), u = bf16(lin(x, w3))
 * each lin with its live LoRA slots (one rank-space pass over x for both).
 * w1 and w3 share n, k, bits and quant mode; h is 16-byte aligned, ldh >= n
 * and a multiple of 8. Replaces: the w1 and w3 lin calls and swiglu of
 * gpu_ff (src/ming-dit.cc:2155-2157; swiglu at src/metal/ming_ops.metal:95-112). */
int mp_linear_swiglu(mp_ctx* ctx, const mp_weight* w1, const mp_weight* w3, const void* x,
                     int64_t ldx, void* h, int64_t ldh, int m, void* stream);

/* `count` attention projections of the same input x (q, k, v) in one launch,
 * each written HEAD-MAJOR: ys[i] is bf16 [n_i / 128][m][128] (16-byte
 * aligned), head width 128, n_i a multiple of 128. For each i with
 * norm_w[i] != NULL (q and k) every head row also gets, before the store,
 *   z = bf16(y * rsqrt(mean(y^2) + eps) * norm_w[i][f])   (y = bf16 projection)
 *   (out[2j], out[2j+1]) = bf16(z[2j] c - z[2j+1] s, z[2j] s + z[2j+1] c)
 * with c = rope_cos[t][j], s = rope_sin[t][j] (f32 [m][64], row t = token row
 * t of x; the caller offsets the tables to the first row; gains and tables
 * 16-byte aligned). norm_w may be NULL
 * (no member normed; then the tables may be NULL). Live LoRA slots as in
 * mp_linear_shared. Replaces: the q/k/v lin calls, the per-head rms, tr_rope
 * and the v transpose of run_block (src/ming-dit.cc:2078-2088; tr_rope at
 * :1885-1894). */
int mp_linear_heads(mp_ctx* ctx, const mp_weight* const* ws, void* const* ys, int count,
                    const void* x, int64_t ldx, int m, const uint16_t* const* norm_w, float eps,
                    const float* rope_cos, const float* rope_sin, void* stream);

/* Non-causal attention, head dim 128, over the head-major q, k, v that
 * mp_linear_heads writes: for head h and query row i < s,
 *   o[i][128h .. 128h + 127] = softmax(scale * q_i . K_h^T) . V_h   (bf16 out)
 * q, k, v: device bf16, head h's s rows of 128 at element offset
 * h * head_stride (0: s * 128, i.e. [nh][s][128]; a batch of images sharing
 * one head-major tensor passes its own first row and the whole tensor's
 * head stride), 16-byte aligned; o: device bf16 [s][ldo], ldo >= 128 * nh
 * and a multiple of 8 (token-major: the to_out projection's input as it
 * is). P is rounded to bf16 for the P.V product; row statistics in f32.
 * Replaces: run_attn over a block's rows and the transpose back to
 * token-major (src/ming-dit.cc:1905-2039, :2090-2092). */
int mp_attention(mp_ctx* ctx, const void* q, const void* k, const void* v, int s, int nh,
                 int64_t head_stride, float scale, void* o, int64_t ldo, void* stream);

/* The sandwich-norm residual step after to_out and after w2, one pass over
 * the rows:
 *   s   = bf16(o * rsqrt(mean(o^2) + eps) * o_gain)         (o != NULL)
 *   x   = bf16(x + tanh(gate) * s)   (gate != NULL)  or  bf16(x + s)
 *   nrm = bf16(x * rsqrt(mean(x^2) + eps) * nrm_gain)       (nrm != NULL)
 * With o == NULL only nrm is computed (x is read, not written). x, o, nrm:
 * device bf16 [m, h], 16-byte aligned, row strides (elements) >= h and
 * multiples of 8; o_gain, gate, nrm_gain: device bf16 [h], 16-byte aligned;
 * h a multiple of 8, at most 8192. The mean is the sum times (1/h).
 * Replaces: rms of the sub-layer output, gated (gated_residual_tanh) or
 * resid into the joint stream, and rms into the next sub-layer's input
 * (src/ming-dit.cc:2096-2101 with :2104, :2256-2261 with the next block's
 * first rms; src/metal/ming_ops.metal:55-93). */
int mp_rms_residual(mp_ctx* ctx, void* x, int64_t ldx, const void* o, int64_t ldo,
                    const void* o_gain, const void* gate, void* nrm, int64_t ldn,
                    const void* nrm_gain, int h, int m, float eps, void* stream);

/* ---- modulation -------------------------------------------------------- */

/* The adaLN Linears of `n_blocks` modulated blocks, prepared for one
 * batched launch. ada[i]: weight [4H, K_ada] (packed or dense); ada_bias[i]:
 * bf16 [4H]; an1[i] / fn1[i]: bf16 [H] norm gains to fold (1 + scale) into,
 * or NULL. Host or device pointers. Replaces: the per-block adaLN weights
 * loaded by load_block_ (src/ming-dit.cc:858-864). */
int mp_modulation_create(mp_ctx* ctx, int n_blocks, const mp_weight* const* ada,
                         const uint16_t* const* ada_bias, const uint16_t* const* an1,
                         const uint16_t* const* fn1, mp_modset** out);
int mp_modulation_free(mp_ctx* ctx, mp_modset* set);
/* mods[b, i, :] = W_b · temb[i] + bias_b (bf16 [n_blocks, m, 4H]);
 * nw1[b, i, :] = an1_b · (1 + mods[b, i, 0:H]), nw3[b, i, :] = fn1_b ·
 * (1 + mods[b, i, 2H:3H]) (bf16 [n_blocks, m, H]; either may be NULL).
 * temb: device bf16 [m, K_ada], m <= 16 (one token per image of a batch;
 * a token's rows are the same bits whatever m is). Replaces: fill_mod
 * (src/ming-dit.cc:2266-2273) for every modulated block at once. */
int mp_modulation_all(mp_ctx* ctx, const mp_modset* set, const void* temb, int m, void* mods,
                      void* nw1, void* nw3, void* stream);

/* ---- pack I/O ------------------------------------------------------------ */

/* A safetensors checkpoint or pack opened for reading: one file, or every
 * *.safetensors file of a directory (shards), memory-mapped; host only (no
 * device needed). Replaces: the WeightSet reads of the DiT's tensors
 * (load_qw_ / load_block_, src/ming-dit.cc:802-864). */
typedef struct mp_pack mp_pack;
typedef struct {
  const char* name;   /* valid while the pack is open */
  const char* dtype;  /* "BF16", "F16", "F32", "U32", ... */
  int32_t ndim;
  int64_t shape[8];
  const void* data;   /* host pointer into the mapped file */
  size_t bytes;
} mp_tensor_info;
int mp_pack_open(const char* path, mp_pack** out);
/* Why the last mp_pack_open / mp_pack_quantize of this thread failed. */
const char* mp_pack_last_error(void);
int mp_pack_close(mp_pack* pack);
int mp_pack_count(const mp_pack* pack);
int mp_pack_tensor_at(const mp_pack* pack, int i, mp_tensor_info* info);
/* MP_EINVAL when the tensor is absent. */
int mp_pack_find(const mp_pack* pack, const char* name, mp_tensor_info* info);
/* A "__metadata__" value, or NULL. */
const char* mp_pack_metadata(const mp_pack* pack, const char* key);
const char* mp_pack_error(const mp_pack* pack);
/* Uploads projection `base` ("layers.3.attention.to_q") as load_qw_ does
 * (src/ming-dit.cc:802-831, detection :1115-1135): packed when
 * `<base>.scales` sits beside `<base>.weight` (U32 codes [N, K*bits/32],
 * scales / biases [N, K/64] narrowed to bf16; no biases = symmetric 8-bit),
 * bits from the shapes (4 or 8); otherwise the dense `<base>.weight`
 * (narrowed to bf16). */
int mp_pack_upload(mp_ctx* ctx, const mp_pack* pack, const char* base, mp_weight** out);
/* Writes a w8 / w4 pack of the dense checkpoint `src` (a .safetensors file,
 * or a directory of shards plus config.json) to `dst` (a file, or a
 * directory created if needed): the reference's selection
 * (src/ming-quant-family.cc:31-59) quantized with per-64-group affine
 * min/max scales and biases (bf16) and codes packed LSB first; every other
 * tensor copied unchanged; config.json gains "quantization": {"bits",
 * "group_size"}. Host only. Counts of quantized / copied tensors in
 * *n_quantized / *n_kept (nullable). Replaces: the host's model-quantize run
 * for this family (tests/ming-quant-test.cc:507-549 pins its selection). */
int mp_pack_quantize(const char* src, const char* dst, int bits, int* n_quantized, int* n_kept);

/* ---- allocation-free projection ---------------------------------------- */

/* No counterpart in the reference. For callers that cannot call cudaMalloc —
 * a host whose memory planner owns every device allocation, or a serving loop
 * where an allocation or free could synchronize the device — this runs one
 * adapter's fused projection, y = x · deq(W)^T + strength · (x a^T) b^T, with
 * the rank-space intermediate in a fixed 4 MiB device array of this library
 * (2 Mi bf16 elements; every GPU that loads the library holds it until the
 * process exits) instead of context scratch. It allocates nothing.
 *   a: device bf16 [rank, k] (alpha folded in), b: device bf16 [n, rank],
 *      both 16-byte aligned; rank a multiple of 8 in [8, 256];
 *   m * roundup(rank, 64) must not exceed 2 Mi elements (else MP_EINVAL);
 *   the slots bound to `w` with mp_lora_bind are NOT applied here;
 *   strength 0 runs the base projection alone.
 * The first call on a device looks up the array's device address (once per
 * device, kept for the process); make that first call before any stream
 * capture. The kept address does not survive cudaDeviceReset: do not call
 * this entry point again in a process that reset the device. The rank-space
 * pre-GEMM runs unsplit (a K split needs fp32 partial sums in memory this
 * entry point does not allocate), so at few rows and a long K (to_out or w2
 * over caption rows) it is slower than mp_linear's. Every call shares
 * the one array and it keeps the last call's contents: calls whose kernels
 * overlap on the GPU (other streams, other contexts on the same device) race
 * on it — order them on one stream. */
int mp_linear_lora_static(mp_ctx* ctx, const mp_weight* w, const void* x, int64_t ldx,
                          const uint16_t* a, const uint16_t* b, int rank, float strength,
                          void* y, int64_t ldy, int m, void* stream);

/* ---- engagement -------------------------------------------------------- */

int mp_engagement_get(const mp_ctx* ctx, mp_engagement* out);
int mp_engagement_reset(mp_ctx* ctx);

#ifdef __cplusplus
}
#endif

#endif /* MINGPROJ_H */
