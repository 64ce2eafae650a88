// Launch parameters shared by the host side of the C-ABI and the sm_100a
// kernels. Everything a launch needs is passed BY VALUE in these structs, so
// the strengths in force when a projection is enqueued are the ones it uses
// (a strength re-set between forwards never races a launch in flight).
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace mp {

constexpr int kMaxSlots = 8;       // LoRA slots (the reference's lora::Stack::kMax)
constexpr int kMaxSegments = 16;   // row segments with their own strength vector
constexpr int kMaxRanges = 32;     // rank-space column ranges (slot runs) per launch

// Pipeline geometry of the projection kernel (CTA pairs, mp_proj.cu).
constexpr int kBlockN = 128;       // output features per CTA (a pair covers 256: MMA M)
constexpr int kBlockK = 64;        // K per stage == one quantization group
constexpr int kMaxTok = 256;       // token rows of one accumulator (MMA N), at most
constexpr int kMaxTileTok = 512;   // token rows per pair tile (two accumulators), at most
constexpr int kEpiRows = 64;       // token rows per epilogue store (the output map's box)
constexpr int kWStageBytes = kBlockN * 128;   // weight tile: codes or bf16
constexpr int kTmemCols = 512;
constexpr int kMaxMembers = 4;     // projections of one input in one launch (q/k/v, w1/w3)
constexpr int kMaxSplits = 16;     // K splits of a split-K launch
constexpr int kHeadDim = 128;      // attention head width (one CTA's features)

// Device-side error word bits (OR-ed by kernels, read by mp_sync_check).
constexpr uint32_t kErrTimeout = 1u;

// Optional epilogue scaling of the rank-space intermediate: the value in
// token row t and rank column j is multiplied by
//   seg_scale[segment(t)][range_slot[range(j)]].
struct EpilogueScale {
  int32_t enabled;
  int32_t n_seg;
  int32_t seg_start[kMaxSegments + 1];     // token row boundaries
  float seg_scale[kMaxSegments][kMaxSlots];
  int32_t n_ranges;
  int32_t range_start[kMaxRanges + 1];     // rank column boundaries
  int32_t range_slot[kMaxRanges];          // slot whose strength scales the range
};

// One projection of a launch: its weight, output and appended LoRA K tiles.
// A launch covers the pairs [pair_begin, next member's pair_begin) for it.
struct ProjMember {
  CUtensorMap tm_w;   // packed codes [N, K*bits/8] u8 (box {64*bits/8, 128}, SW64/SW32)
                      // or bf16 [N, K] (box {64, 128}, SW128)
  CUtensorMap tm_t;   // rank-space intermediate [M, R] bf16 (box {64, sub/2}, SW128)
  CUtensorMap tm_b;   // stacked LoRA B [N, R] bf16 (box {64, 128}, SW128)
  CUtensorMap tm_y;   // output [M, N] bf16 (box {64, 32} for 256/512-token tiles, else
                      // {64, kEpiRows}; SW128)
  const uint32_t* sb; // per row, per group: bf16 scale (low half) | bf16 bias (high half)
  int32_t N;
  int32_t bits;       // 0 dense bf16, 4 or 8 packed codes
  int32_t sb_stride;  // u32 per row of `sb` (multiple of 4)
  int32_t lora_ktiles;  // extra 64-wide K tiles taken from (tm_t, tm_b)
  uint32_t code_xor;  // 0x80808080 turns signed 8-bit codes into offset-binary
  float code_offset;  // 32768 + the codes' zero point (128 for signed 8-bit codes, else 0)
  int32_t pair_begin;
  int32_t t_col;      // first column of this member's ranks in the rank-space intermediate
  // SwiGLU pair (swiglu = 1): the member is h = silu(x·W1^T) ⊙ (x·W3^T) with
  // N = the FFN width. Each CTA holds 64 rows of W1 (tm_w, sb) and the same
  // 64 rows of W3 (tm_w3, sb3), both maps with 64-row boxes; a pair tile covers
  // 128 output features; tm_b is the row-interleaved LoRA B stack
  // [B1 rows 64b.. ‖ 0 ; 0 ‖ B3 rows 64b..] per 64-feature block b, over the
  // ranks [T1 | T3]; tm_y is h.
  int32_t swiglu;
  CUtensorMap tm_w3;
  const uint32_t* sb3;
  // Attention-head member (heads = 1; N a multiple of kHeadDim): each CTA's
  // 128 features are one head, and tm_y is the head-major output
  // [N / kHeadDim][M][kHeadDim] bf16 (3-D map, box {64, 32, 1}). With
  // head_norm = 1 the epilogue first applies the head's RMSNorm (gain
  // norm_w[kHeadDim] bf16, norm_eps) and the interleaved-pair rotary
  // embedding (rope_cos / rope_sin f32 [M][kHeadDim / 2], row = token row).
  int32_t heads;
  int32_t head_norm;
  float norm_eps;
  const uint16_t* norm_w;
  const float* rope_cos;
  const float* rope_sin;
};

struct ProjParams {
  CUtensorMap tm_x;   // activations [M, K] bf16 (box {64, sub/2}, SW128), shared by all members
  int32_t M, K;
  int32_t n_tok;      // token rows per pair tile: 64, 128, 256 or 512 (two accumulators)
  int32_t n_members;
  int32_t n_pairs;    // feature pairs of the launch (all members)
  int32_t n_ttiles;   // token tiles: ceil(M / n_tok)
  int32_t n_tiles;    // n_pairs * n_ttiles * max(ksplit, 1): the persistent grid's work list
  // Order of the work list within a K split: tile_group <= 1 walks token
  // tiles fastest (feature pair after feature pair); tile_group = G > 1 takes
  // the feature pairs in groups of G, and within a group the pair fastest,
  // then the token tile, so the tiles running at one time share a few x
  // tiles (each read from memory once per group) and G pairs' weights.
  int32_t tile_group;
  uint64_t wait_limit_ns;
  uint32_t* err;      // device error word
  EpilogueScale scale;  // rank-space pre-GEMM / prologue only
  // Split-K (ksplit > 1, a single member): the tiles of split z run the K tiles
  // [z * kt_per_split, min((z + 1) * kt_per_split, K tiles)) (the last split
  // also takes the member's LoRA K tiles) and writes its fp32 partial sums,
  // unscaled, to part[z][t][f] (row stride part_ld) instead of the bf16
  // output; lora_reduce_kernel adds the splits in z order.
  int32_t ksplit;
  int32_t kt_per_split;
  float* part;
  int32_t part_ld;
  // With lora_apart != 0 the appended LoRA K tiles are a split of their own:
  // splits z < ksplit - 1 run base K tiles only, split ksplit - 1 runs only
  // the LoRA K tiles (its partial sums are T·B_stack^T). A launch runs the
  // splits [z_first, z_first + z_count) (z_count 0: all of them), so the
  // LoRA split can go in a launch of its own once T is ready.
  int32_t lora_apart;
  int32_t z_first;
  int32_t z_count;
  // Fused rank-space prologue (n_pre > 0): before their member tiles, the
  // pairs with the fewest member tiles run n_pre prologue units, each the
  // full-K product of 512 token rows x 256 rank rows of T = scale ⊙ (x ·
  // A_stack^T) (member `pre`: the stacked A as a dense weight, tm_y = T),
  // stored scaled in bf16; each CTA of the unit then sets its flag
  // flags[(rank_pair * pre_ttiles + token_tile) * 2 + cta] = epoch. A member
  // tile waits for the flags of its T rows before its appended LoRA K tiles.
  // The launch is cooperative (every pair resident), so the waits end.
  int32_t n_pre;
  int32_t pre_ttiles;     // 512-token tiles of the prologue: ceil(M / 512)
  int32_t pre_rpairs;     // 256-row rank pairs: ceil(R / 256)
  uint32_t* flags;
  uint32_t epoch;
  ProjMember pre;
  ProjMember mem[kMaxMembers];
};

constexpr int kPreTok = 512;  // token rows of a prologue unit (two accumulators, as member tiles)

// Second pass of a split-K launch: out[t, j] = bf16(scale(t, j) * sum_z
// part[z][t][j]) for t < M, j < R, the splits added in z order (the result
// does not depend on launch timing). `scale` as in EpilogueScale; with
// enabled == 0 the sum is stored unscaled.
struct ReduceParams {
  const float* part;
  int32_t ksplit, M, R, part_ld;
  uint16_t* out;
  int32_t out_ld;
  EpilogueScale scale;
};

// Batched adaLN modulation: for every block b and token m,
//   mods[b, m, :] = bf16(W_b · temb[m] + bias_b)
//   nw1[b, m, i] = bf16(an1_b[i] · (1 + mods[b, m, i]))          (chunk 0)
//   nw3[b, m, i] = bf16(fn1_b[i] · (1 + mods[b, m, 2H + i]))     (chunk 2)
struct ModBlock {
  const uint8_t* w;      // codes [N, K*bits/8] or bf16 [N, K]
  const uint32_t* sb;    // (scale | bias << 16) per group, stride sb_stride
  const uint16_t* bias;  // bf16 [N]
  const uint16_t* an1;   // bf16 [H] or null
  const uint16_t* fn1;   // bf16 [H] or null
};

struct ModParams {
  const ModBlock* blocks;  // device array [n_blocks]
  int32_t n_blocks;
  int32_t N, K, H;         // N == 4 * H
  int32_t bits;
  uint32_t code_xor;
  float code_magic;
  int32_t sb_stride;
  int32_t M;               // tokens of this launch (<= 8; <= kModMaxTok off the lane path)
  int32_t m_stride;        // tokens per block in the output arrays (>= M)
  const uint16_t* temb;    // bf16 [M, K]
  uint16_t* mods;          // bf16 [n_blocks, m_stride, N] (token 0 of this launch)
  uint16_t* nw1;           // bf16 [n_blocks, m_stride, H] or null
  uint16_t* nw3;           // bf16 [n_blocks, m_stride, H] or null
  // per block: its weight rows [N, K] as a 2-D tensor map with 128-byte x
  // 32-row boxes and the 128-byte swizzle (lane-per-row path)
  const CUtensorMap* maps;
  uint32_t* err;           // device error word
  uint64_t wait_limit_ns;
};

constexpr int kModMaxTok = 4;      // tokens of one generic-path launch (registers scale with it)
constexpr int kModMaxBatch = 16;   // tokens of one mp_modulation_all call (several launches)

// The sandwich-norm residual step (mp_norm.cu), per token row r < M:
//   s   = bf16(o * rsqrt(mean(o^2) + eps) * o_gain)          (o != null)
//   x   = bf16(x + tanh(gate) * s)  (gate != null)  or  bf16(x + s)
//   nrm = bf16(x * rsqrt(mean(x^2) + eps) * nrm_gain)        (nrm != null)
// bf16 rows of H (a multiple of 8, at most kNormMaxH); row strides in elements.
constexpr int kNormMaxH = 8192;

// Non-causal attention over head-major q, k, v (mp_attn.cu): for head h and
// query row i < S,  o[i, 128h .. 128h + 127] = softmax(scale · q_i · K^T) · V.
// tm_q / tm_k / tm_v: bf16 [NH][S][128] as 3-D maps {128, S, NH}, boxes
// {64, 128, 1} (q, v) and {64, 64, 1} (k), 128-byte swizzle (rows past S read
// zeros). o: bf16 [S][ldo].
struct AttnParams {
  CUtensorMap tm_q;
  CUtensorMap tm_k;
  CUtensorMap tm_v;
  uint16_t* o;
  int64_t ldo;
  int32_t S, NH;
  float scale_log2;  // softmax scale · log2(e)
  uint64_t wait_limit_ns;
  uint32_t* err;
};
struct RmsResidualParams {
  uint16_t* x;
  int64_t ldx;
  const uint16_t* o;
  int64_t ldo;
  const uint16_t* o_gain;
  const uint16_t* gate;
  uint16_t* nrm;
  int64_t ldn;
  const uint16_t* nrm_gain;
  int32_t M, H;
  float eps;
};

}  // namespace mp
