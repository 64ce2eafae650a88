// Host side of the mingproj C-ABI (include/mingproj.h): contexts, weight
// upload, LoRA slot binding and the stacked-adapter cache, launch assembly
// for the projection and modulation kernels, engagement counters.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/mingproj.h"
#include "mp_kernels.h"

namespace mp {
cudaError_t launch_proj_pair(const ProjParams& p, cudaStream_t stream);
cudaError_t launch_lora_reduce(const ReduceParams& p, cudaStream_t stream);
int resident_pairs();
int pick_ntok_pair(int m, int pairs);
cudaError_t launch_wait_selftest(uint64_t limit_ns, uint32_t* err, cudaStream_t stream);
cudaError_t launch_mod(const ModParams& p, cudaStream_t stream);
int mod_tokens_per_launch(int n, int k, int n_blocks);
cudaError_t launch_rms_residual(const RmsResidualParams& p, cudaStream_t stream);
cudaError_t launch_attention(const AttnParams& p, cudaStream_t stream);
}  // namespace mp

using mp::ProjParams;

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  }
  return fn;
}

struct Stack {
  bool valid = false;
  uint32_t mask = 0;       // live slots the stack was built for
  uint64_t bind_version = 0;
  int rpad = 0;            // stacked rank, padded to 64
  int ranks[mp::kMaxSlots] = {};
  uint16_t* a = nullptr;   // [rpad, k]
  size_t a_cap = 0;
  uint16_t* b = nullptr;   // [n, rpad]
  size_t b_cap = 0;
  CUtensorMap tm_a;        // box {64, 128}, SW128 (LoRA-down "weight")
  CUtensorMap tm_b;        // box {64, 128}, SW128 (appended K tiles)
  uint64_t version = 0;
};

}  // namespace

struct mp_weight {
  mp_weight_desc d{};
  void* w = nullptr;       // codes bytes [n, k*bits/8] or bf16 [n, kp]
  size_t w_bytes = 0;      // algorithmic bytes (no padding)
  int kp = 0;              // row pitch in elements of dense weights / LoRA A rows: k rounded up to 8
  uint32_t* sb = nullptr;  // [n, sb_stride] (bf16 scale | bf16 bias << 16)
  int sb_stride = 0;
  CUtensorMap tm_w;
  CUtensorMap tm_w64;      // the same rows with 64-row boxes (SwiGLU pairs), built on first use
  bool has_w64 = false;
  int rank[mp::kMaxSlots] = {};
  uint16_t* la[mp::kMaxSlots] = {};  // [rank, k]
  uint16_t* lb[mp::kMaxSlots] = {};  // [n, rank]
  uint64_t bind_version = 1;
  Stack stack;
};

struct mp_modset {
  int n_blocks = 0;
  int n = 0, k = 0, bits = 0, mode = 0, sb_stride = 0;
  mp::ModBlock* dev_blocks = nullptr;
  CUtensorMap* dev_maps = nullptr;  // per block: weight rows, 128-byte x 32-row boxes
  std::vector<void*> owned;  // bias / gain copies
};

namespace {

struct SharedStack {
  std::vector<uint64_t> versions;
  uint16_t* a = nullptr;
  size_t a_cap = 0;
  int rtot = 0;
  CUtensorMap tm_a;
  // SwiGLU pairs: the two members' B stacks interleaved per 64 features,
  // [B1 rows 64b.. | 0 ; 0 | B3 rows 64b..] over the ranks [T1 | T3]
  std::vector<uint64_t> bc_versions;
  uint16_t* bc = nullptr;
  size_t bc_cap = 0;
  CUtensorMap tm_bc;
};

}  // namespace

struct mp_ctx {
  int device = 0;
  std::string err = "";
  float strength[mp::kMaxSlots];
  int image_rows = 0;  // rows of one image per launch (0: the launch, or its longest segment)
  int n_seg = 0;
  int32_t seg_start[mp::kMaxSegments + 1] = {};
  float seg_scale[mp::kMaxSegments][mp::kMaxSlots] = {};
  uint32_t* err_word = nullptr;
  uint16_t* scratch = nullptr;  // rank-space intermediate
  size_t scratch_cap = 0;       // elements
  float* part = nullptr;        // split-K partial sums (pre-GEMM or projection)
  size_t part_cap = 0;          // elements
  // A split-K projection with live slots runs its rank-space pre-GEMM and the
  // LoRA split on a side stream, beside the base splits: that chain's
  // partial sums, the stream and its fork / join events.
  float* part_side = nullptr;
  size_t part_side_cap = 0;
  cudaStream_t side = nullptr;
  cudaEvent_t ev_fork = nullptr;
  cudaEvent_t ev_join = nullptr;
  uint32_t* flags = nullptr;    // fused-prologue ready flags (zeroed on allocation)
  size_t flags_cap = 0;         // entries
  uint32_t epoch = 0;           // value of a flag that is set, per fused launch
  bool fuse_off = false;        // cooperative launches refused on this device
  // Set once a call was made while its stream was being captured into a CUDA
  // graph: from then on the graph may hold this context's buffers, so a
  // buffer that has to grow is retired (freed at destroy), never freed.
  bool captured = false;
  std::vector<void*> retired;
  // Bumped by every change that alters what a launch computes (a strength,
  // the row segments, a LoRA binding): a captured graph holds the values of
  // its capture and is stale once this moves.
  uint64_t state_version = 0;
  uint64_t wait_limit_ns = 2000000000ull;
  mp_engagement eng{};
  std::map<std::vector<uintptr_t>, SharedStack> shared;
};

namespace {

int fail(mp_ctx* c, int code, const char* fmt, ...) {
  if (c != nullptr) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    c->err = buf;
  }
  return code;
}

int cuda_fail(mp_ctx* c, cudaError_t e, const char* what) {
  return fail(c, e == cudaErrorMemoryAllocation ? MP_ENOMEM : MP_ECUDA, "%s: %s", what,
              cudaGetErrorString(e));
}

#define MP_CUDA(ctx, call)                               \
  do {                                                   \
    cudaError_t e_ = (call);                             \
    if (e_ != cudaSuccess) return cuda_fail(ctx, e_, #call); \
  } while (0)

int use_device(mp_ctx* c) {
  cudaError_t e = cudaSetDevice(c->device);
  if (e != cudaSuccess) return cuda_fail(c, e, "cudaSetDevice");
  return MP_OK;
}

bool encode_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner,
               uint64_t outer, uint64_t stride_bytes, uint32_t box_inner, uint32_t box_outer,
               CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Token rows of one epilogue store box: 32 with the token-row accumulators of
// 256- and 512-token tiles (each epilogue warp stores its own 32 rows), 64
// with the feature-row accumulators of narrower tiles.
int epi_box_rows(int ntok) { return ntok >= mp::kMaxTok ? 32 : mp::kEpiRows; }

// Output map for the pair kernel's bulk stores: [m, n] bf16 rows of ldy,
// box = 64 features x one pair token tile, 128-byte swizzle.
bool encode_y(CUtensorMap* m, const void* y, int64_t ldy, int n, int rows, int ntok) {
  return encode_2d(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, y, static_cast<uint64_t>(n),
                   static_cast<uint64_t>(rows), static_cast<uint64_t>(ldy) * 2, 64,
                   static_cast<uint32_t>(ntok), CU_TENSOR_MAP_SWIZZLE_128B);
}

// Head-major output map of an attention-head member: [n / 128][rows][128]
// bf16, box = 64 features x 64 tokens of one head, 128-byte swizzle (the
// same staging layout as encode_y's boxes).
bool encode_heads_y(CUtensorMap* m, const void* y, int n, int rows, int ntok) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  const uint64_t hd = mp::kHeadDim;
  cuuint64_t dims[3] = {hd, static_cast<uint64_t>(rows), static_cast<uint64_t>(n) / hd};
  cuuint64_t strides[2] = {hd * 2, static_cast<uint64_t>(rows) * hd * 2};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(epi_box_rows(ntok)), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(y), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Token rows of one accumulator (MMA N) for a pair tile of `ntok` rows: the
// TMA boxes of x, the rank-space intermediate and y are sized by it.
int sub_tok(int ntok) { return std::min(ntok, mp::kMaxTok); }

// Feature pairs (256 output rows) a projection of n outputs occupies.
int pairs_of(int n) { return (n + 2 * mp::kBlockN - 1) / (2 * mp::kBlockN); }

// Rows of one image of an m-row call: mp_set_image_rows' count, else the
// longest row segment (mp_set_strengths_rows) when the call holds several
// images, else m. Every choice that changes a row's accumulation order (token
// tile, K splits of the projection and of its rank-space pre-GEMM) is made
// from this count, so a batch of equal-length images has each image's bits of
// its own call.
int image_rows(const mp_ctx* c, int m) {
  if (c->image_rows > 0) return std::min(c->image_rows, m);
  if (c->n_seg <= 1) return m;
  int most = 0;
  for (int g = 0; g < c->n_seg; ++g) {
    const int lo = std::min(std::max(c->seg_start[g], 0), m);
    const int hi = std::min(std::max(c->seg_start[g + 1], lo), m);
    most = std::max(most, hi - lo);
  }
  return most > 0 ? most : m;
}

uint32_t live_mask(const mp_ctx* c, const mp_weight* w) {
  uint32_t mask = 0;
  for (int i = 0; i < mp::kMaxSlots; ++i) {
    if (w->rank[i] <= 0) continue;
    bool live = false;
    if (c->n_seg > 0) {
      for (int g = 0; g < c->n_seg; ++g) live = live || c->seg_scale[g][i] != 0.0f;
    } else {
      live = c->strength[i] != 0.0f;
    }
    if (live) mask |= 1u << i;
  }
  return mask;
}

// True while `stream` is being captured into a CUDA graph (also marks the
// context as captured). Kernels launched then are replayed later with the
// parameters they had at capture, so a launch whose correctness rests on a
// per-launch host value (the fused prologue's epoch) puts what makes it safe
// on replay into the graph too.
bool capturing(mp_ctx* c, cudaStream_t stream) {
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &st) != cudaSuccess) {
    (void)cudaGetLastError();
    st = cudaStreamCaptureStatusActive;  // the legacy stream while another captures
  }
  if (st == cudaStreamCaptureStatusNone) return false;
  c->captured = true;
  return true;
}

template <class T>
int ensure_buf(mp_ctx* c, T** p, size_t* cap, size_t elems, cudaStream_t stream) {
  if (*cap >= elems && *p != nullptr) return MP_OK;
  if (*p != nullptr) {
    if (capturing(c, stream) || c->captured) {
      // a graph may read the old buffer on replay: keep it until destroy
      // (no synchronisation and no free are allowed during a capture)
      c->retired.push_back(*p);
    } else {
      cudaStreamSynchronize(stream);
      // the side stream's LoRA chain may still read or write context buffers
      if (c->side != nullptr) cudaStreamSynchronize(c->side);
      cudaFree(*p);
    }
    *p = nullptr;
    *cap = 0;
  }
  void* q = nullptr;
  // an allocation is not a stream operation; a capture in global mode would
  // still refuse it from this thread unless the thread's mode is relaxed
  cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
  cudaThreadExchangeStreamCaptureMode(&mode);
  cudaError_t e = cudaMalloc(&q, std::max<size_t>(elems, 1) * sizeof(T));
  cudaThreadExchangeStreamCaptureMode(&mode);
  if (e != cudaSuccess) return cuda_fail(c, e, "cudaMalloc");
  *p = static_cast<T*>(q);
  *cap = elems;
  return MP_OK;
}

// Ready flags of fused prologues: at least `n` entries, zeroed when (re)allocated.
int ensure_flags(mp_ctx* c, size_t n, cudaStream_t stream) {
  if (c->flags_cap >= n && c->flags != nullptr) return MP_OK;
  const size_t cap = std::max<size_t>(n, 1024);
  int rc = ensure_buf(c, &c->flags, &c->flags_cap, cap, stream);
  if (rc != MP_OK) return rc;
  MP_CUDA(c, cudaMemsetAsync(c->flags, 0, cap * sizeof(uint32_t), stream));
  return MP_OK;
}

// The side stream and fork / join events of the concurrent LoRA chain,
// created on first use (the context's device is current).
int ensure_side(mp_ctx* c) {
  if (c->side != nullptr && c->ev_fork != nullptr && c->ev_join != nullptr) return MP_OK;
  // not stream operations; relaxed, so a first use inside a capture in
  // global mode is not refused
  cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
  cudaThreadExchangeStreamCaptureMode(&mode);
  cudaError_t e = cudaSuccess;
  if (c->side == nullptr) e = cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking);
  if (e == cudaSuccess && c->ev_fork == nullptr)
    e = cudaEventCreateWithFlags(&c->ev_fork, cudaEventDisableTiming);
  if (e == cudaSuccess && c->ev_join == nullptr)
    e = cudaEventCreateWithFlags(&c->ev_join, cudaEventDisableTiming);
  cudaThreadExchangeStreamCaptureMode(&mode);
  if (e != cudaSuccess) return cuda_fail(c, e, "side stream / events");
  return MP_OK;
}

// Builds (or reuses) the stacked factors of the live slots of `w`, in slot
// order: A rows [r_0 | r_1 | ...] padded with zero rows to a multiple of 64,
// B columns in the same order, zero-padded.
int ensure_stack(mp_ctx* c, mp_weight* w, uint32_t mask, cudaStream_t stream) {
  Stack& st = w->stack;
  if (st.valid && st.mask == mask && st.bind_version == w->bind_version) return MP_OK;
  const int n = w->d.n, k = w->d.k, kp = w->kp;
  int rtot = 0;
  for (int i = 0; i < mp::kMaxSlots; ++i)
    if (mask & (1u << i)) rtot += w->rank[i];
  const int rpad = (rtot + 63) / 64 * 64;
  int rc = ensure_buf(c, &st.a, &st.a_cap, static_cast<size_t>(rpad) * kp, stream);
  if (rc != MP_OK) return rc;
  rc = ensure_buf(c, &st.b, &st.b_cap, static_cast<size_t>(n) * rpad, stream);
  if (rc != MP_OK) return rc;
  MP_CUDA(c, cudaMemsetAsync(st.a, 0, static_cast<size_t>(rpad) * kp * 2, stream));
  MP_CUDA(c, cudaMemsetAsync(st.b, 0, static_cast<size_t>(n) * rpad * 2, stream));
  int off = 0;
  for (int i = 0; i < mp::kMaxSlots; ++i) {
    st.ranks[i] = 0;
    if (!(mask & (1u << i))) continue;
    const int r = w->rank[i];
    st.ranks[i] = r;
    MP_CUDA(c, cudaMemcpy2DAsync(st.a + static_cast<size_t>(off) * kp,
                                 static_cast<size_t>(kp) * 2, w->la[i],
                                 static_cast<size_t>(k) * 2, static_cast<size_t>(k) * 2, r,
                                 cudaMemcpyDeviceToDevice, stream));
    MP_CUDA(c, cudaMemcpy2DAsync(st.b + off, static_cast<size_t>(rpad) * 2, w->lb[i],
                                 static_cast<size_t>(r) * 2, static_cast<size_t>(r) * 2, n,
                                 cudaMemcpyDeviceToDevice, stream));
    off += r;
  }
  if (rpad > 0) {
    if (!encode_2d(&st.tm_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, st.a, k, rpad,
                   static_cast<uint64_t>(kp) * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_2d(&st.tm_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, st.b, rpad, n,
                   static_cast<uint64_t>(rpad) * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B))
      return fail(c, MP_ECUDA, "tensor map encode failed (LoRA stack)");
  }
  st.rpad = rpad;
  st.mask = mask;
  st.bind_version = w->bind_version;
  st.valid = true;
  // process-wide, never repeated: a weight freed and another uploaded at the
  // same address can never match a cached shared stack built from the first
  static std::atomic<uint64_t> g_stack_version{0};
  st.version = ++g_stack_version;
  return MP_OK;
}

void fill_scale(const mp_ctx* c, mp::EpilogueScale* es) {
  es->enabled = 1;
  if (c->n_seg > 0) {
    es->n_seg = c->n_seg;
    for (int g = 0; g <= c->n_seg; ++g) es->seg_start[g] = c->seg_start[g];
    for (int g = 0; g < c->n_seg; ++g)
      for (int i = 0; i < mp::kMaxSlots; ++i) es->seg_scale[g][i] = c->seg_scale[g][i];
  } else {
    es->n_seg = 1;
    es->seg_start[0] = 0;
    es->seg_start[1] = INT_MAX;
    for (int i = 0; i < mp::kMaxSlots; ++i) es->seg_scale[0][i] = c->strength[i];
  }
}

// Appends the slot ranges of one stack starting at rank column `base`.
bool add_ranges(mp::EpilogueScale* es, const Stack& st, int base) {
  int off = base;
  for (int i = 0; i < mp::kMaxSlots; ++i) {
    if (!(st.mask & (1u << i))) continue;
    if (es->n_ranges >= mp::kMaxRanges) return false;
    es->range_start[es->n_ranges] = off;
    es->range_slot[es->n_ranges] = i;
    off += st.ranks[i];
    es->range_start[es->n_ranges + 1] = off;
    es->n_ranges += 1;
  }
  return true;
}

int check_y(mp_ctx* c, const void* y, int64_t ldy, int n) {
  if (y == nullptr) return fail(c, MP_EINVAL, "y is NULL");
  if (reinterpret_cast<uintptr_t>(y) % 16 != 0)
    return fail(c, MP_EINVAL, "y must be 16-byte aligned");
  if (ldy < n || ldy % 8 != 0)
    return fail(c, MP_EINVAL, "ldy must be >= n and a multiple of 8 (got %lld)",
                static_cast<long long>(ldy));
  return MP_OK;
}

int check_x(mp_ctx* c, const void* x, int64_t ldx, int k, int m) {
  if (x == nullptr) return fail(c, MP_EINVAL, "x is NULL");
  if (m <= 0) return fail(c, MP_EINVAL, "m must be positive (got %d)", m);
  if (reinterpret_cast<uintptr_t>(x) % 16 != 0)
    return fail(c, MP_EINVAL, "x must be 16-byte aligned");
  if (ldx < k || ldx % 8 != 0)
    return fail(c, MP_EINVAL, "ldx must be >= k and a multiple of 8 (got %lld)",
                static_cast<long long>(ldx));
  return MP_OK;
}

void base_params(const mp_ctx* c, ProjParams* p) {
  std::memset(p, 0, sizeof(*p));
  p->wait_limit_ns = c->wait_limit_ns;
  p->err = c->err_word;
}

// The appended LoRA K tiles of one member: `rpad` rank columns of the
// rank-space intermediate at `tbase` (row stride t_ld), against `tm_b`.
struct LoraTiles {
  int rpad = 0;
  const uint16_t* tbase = nullptr;
  int t_ld = 0;
  const CUtensorMap* tm_b = nullptr;
};

// One projection (weight `w`, or a dense bf16 "weight" map for the
// rank-space pre-GEMM) as member `i` of a launch.
int fill_member(mp_ctx* c, ProjParams* p, int i, const CUtensorMap& tm_w, const uint32_t* sb,
                int sb_stride, int n, int bits, int mode, void* y, int64_t ldy,
                const LoraTiles& lt) {
  mp::ProjMember& mb = p->mem[i];
  mb.tm_w = tm_w;
  mb.sb = sb;
  mb.sb_stride = sb_stride;
  mb.N = n;
  mb.bits = bits;
  const bool sym = bits == 8 && mode == MP_QUANT_SYMMETRIC;
  mb.code_xor = sym ? 0x80808080u : 0u;
  mb.code_offset = sym ? 32896.0f : 32768.0f;
  if (!encode_y(&mb.tm_y, y, ldy, n, p->M, epi_box_rows(p->n_tok)))
    return fail(c, MP_ECUDA, "tensor map encode failed (output)");
  mb.lora_ktiles = 0;
  if (lt.rpad > 0) {
    mb.lora_ktiles = lt.rpad / 64;
    if (!encode_2d(&mb.tm_t, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, lt.tbase, lt.rpad, p->M,
                   static_cast<uint64_t>(lt.t_ld) * 2, 64, static_cast<uint32_t>(sub_tok(p->n_tok) / 2),
                   CU_TENSOR_MAP_SWIZZLE_128B))
      return fail(c, MP_ECUDA, "tensor map encode failed (rank-space intermediate)");
    mb.tm_b = *lt.tm_b;
  }
  return MP_OK;
}

// Order of a launch's work list (ProjParams::tile_group) from the bytes it
// streams: token tile fastest while x fits comfortably in L2 (each weight tile
// is read once, x stays resident); otherwise feature pair fastest, over the
// whole launch when its weights fit in L2 (x streams exactly once) or in
// groups of 16 pairs (x streams once per group, each group's weights stay
// resident).
int tile_group_for(double x_bytes, double w_bytes, int pairs) {
#ifdef MP_FORCE_TILE_GROUP
  (void)x_bytes;
  (void)w_bytes;
  return MP_FORCE_TILE_GROUP > 0 ? std::min(MP_FORCE_TILE_GROUP, pairs) : pairs;
#else
  constexpr double kResident = 48.0 * 1024 * 1024;
  if (x_bytes <= kResident) return 1;
  if (w_bytes <= kResident) return pairs;
  return std::min(16, pairs);
#endif
}

// Sets the launch-wide fields for `count` members whose output widths are
// `ns`, choosing the token tile from the total pair count; `w_bytes` are the
// bytes of the members' weights (codes or bf16) the launch streams.
int begin_launch(mp_ctx* c, ProjParams* p, const void* x, int64_t ldx, int k, int m,
                 const int* ns, int count, double w_bytes, int n_tok = 0) {
  base_params(c, p);
  int pairs = 0;
  for (int i = 0; i < count; ++i) {
    p->mem[i].pair_begin = pairs;
    pairs += pairs_of(ns[i]);
  }
  p->n_members = count;
  p->n_pairs = pairs;
  p->M = m;
  p->K = k;
  p->n_tok = n_tok > 0 ? n_tok : mp::pick_ntok_pair(image_rows(c, m), pairs);
  p->tile_group = tile_group_for(2.0 * m * static_cast<double>(k), w_bytes, pairs);
  if (!encode_2d(&p->tm_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, k, m,
                 static_cast<uint64_t>(ldx) * 2, 64, static_cast<uint32_t>(sub_tok(p->n_tok) / 2),
                 CU_TENSOR_MAP_SWIZZLE_128B))
    return fail(c, MP_ECUDA, "tensor map encode failed (x)");
  return MP_OK;
}

int run_launch(mp_ctx* c, const ProjParams& p, cudaStream_t stream, const char* what) {
  cudaError_t e = mp::launch_proj_pair(p, stream);
  if (e != cudaSuccess) return cuda_fail(c, e, what);
  c->eng.kernels += 1;
  return MP_OK;
}

// Engagement of one projection launched as a member.
void count_projection(mp_ctx* c, const mp_weight* w, int m, const int* ranks) {
  const int n = w->d.n, k = w->d.k;
  c->eng.linear_calls += 1;
  if (w->d.bits == 8) c->eng.gemm_w8 += 1;
  else if (w->d.bits == 4) c->eng.gemm_w4 += 1;
  else c->eng.gemm_dense += 1;
  double flops = 2.0 * m * n * static_cast<double>(k);
  double bytes = static_cast<double>(w->w_bytes) + static_cast<double>(n) * (k / 64) * 4.0 +
                 2.0 * m * k + 2.0 * m * n;
  bool lora = false;
  if (ranks != nullptr) {
    for (int i = 0; i < mp::kMaxSlots; ++i) {
      if (ranks[i] <= 0) continue;
      lora = true;
      flops += 2.0 * m * ranks[i] * static_cast<double>(k + n);
      bytes += 2.0 * ranks[i] * static_cast<double>(k + n);
    }
  }
  if (lora) c->eng.lora_proj += 1;
  c->eng.flops += flops;
  c->eng.bytes += bytes;
}

}  // namespace

namespace mp {

struct SplitChoice {
  int n_tok;
  int ksplit;
  double us;  // modelled time, pre-GEMM and reduce
};

// Token tile and K splits of a rank-space pre-GEMM of `pairs` feature pairs
// over m rows and `base_kt` 64-wide K tiles (r rank columns): the pair with
// the least modelled time. A 64-wide K stage takes ~890 cycles on a
// 256-token tile and ~1250 on a 512-token tile, a CTA adds ~6000 cycles of
// set-up and epilogue, 74 pairs run at once (one CTA per SM), and the second
// pass of a split launch costs ~2 us plus its traffic at ~4 TB/s. At most
// `max_split` splits.
// With room_pairs > 0 only the choices whose splits leave room for one more
// split's tiles beside them within room_pairs CTA pairs are considered.
SplitChoice choose_ksplit(int m, int pairs, int base_kt, int r, int max_split = kMaxSplits,
                          int room_pairs = 0) {
  SplitChoice best{kMaxTok, 1, 0.0};
  double best_us = 1e300;
  for (int nt : {kMaxTileTok, kMaxTok}) {
    const double stage_cycles = nt > kMaxTok ? 1250.0 : 890.0;
    const long long tiles = (m + nt - 1) / nt;
    for (int s = 1; s <= max_split && s <= base_kt; ++s) {
      const int kps = (base_kt + s - 1) / s;
      if ((base_kt + kps - 1) / kps != s) continue;  // every split gets at least one tile
      if (room_pairs > 0 && pairs * tiles * (s + 1) > room_pairs) continue;
      const long long waves = (pairs * tiles * s + 73) / 74;
      double us = static_cast<double>(waves) * (kps * stage_cycles + 6000.0) / 1900.0;
      if (s > 1) us += 2.0 + (static_cast<double>(s) * 4.0 + 2.0) * m * r / 4.0e6;
      if (us < best_us - 1e-9) {
        best_us = us;
        best = SplitChoice{nt, s, us};
      }
    }
  }
  return best;
}

}  // namespace mp

namespace {

// Rank-space pre-GEMM: T[m, 0:rtot] = scale ⊙ (x · A^T), into ctx scratch.
// When the K loop is split, each split writes fp32 partial sums and
// lora_reduce_kernel adds them (in split order), scales and rounds. The split
// count comes from one image's rows (at most max_split); with `side` the
// partial sums go to the side chain's buffer, which the caller has sized.
int launch_lora_down(mp_ctx* c, const CUtensorMap& tm_a, int rtot, const mp::EpilogueScale& es,
                     const void* x, int64_t ldx, int k, int m, cudaStream_t stream,
                     int max_split = mp::kMaxSplits, bool side = false) {
  const int base_kt = (k + mp::kBlockK - 1) / mp::kBlockK;
  const mp::SplitChoice sc =
      mp::choose_ksplit(image_rows(c, m), pairs_of(rtot), base_kt, rtot, max_split);
  const int ks = sc.ksplit;
  ProjParams p;
  int rc = begin_launch(c, &p, x, ldx, k, m, &rtot, 1, 2.0 * rtot * k, sc.n_tok);
  if (rc != MP_OK) return rc;
  p.scale = es;
  rc = fill_member(c, &p, 0, tm_a, nullptr, 0, rtot, 0, 0, c->scratch, rtot, LoraTiles{});
  if (rc != MP_OK) return rc;
  float* part = c->part;
  if (ks > 1) {
    if (side) {
      if (c->part_side_cap < static_cast<size_t>(ks) * m * rtot)
        return fail(c, MP_EINVAL, "side partial-sum buffer too small");
      part = c->part_side;
    } else {
      rc = ensure_buf(c, &c->part, &c->part_cap, static_cast<size_t>(ks) * m * rtot, stream);
      if (rc != MP_OK) return rc;
      part = c->part;
    }
    p.ksplit = ks;
    p.kt_per_split = (base_kt + ks - 1) / ks;
    p.part = part;
    p.part_ld = rtot;
  }
  rc = run_launch(c, p, stream, "proj_pair_kernel (rank-space pre-GEMM)");
  if (rc != MP_OK) return rc;
  if (ks > 1) {
    mp::ReduceParams rp;
    std::memset(&rp, 0, sizeof(rp));
    rp.part = part;
    rp.ksplit = ks;
    rp.M = m;
    rp.R = rtot;
    rp.part_ld = rtot;
    rp.out = c->scratch;
    rp.out_ld = rtot;
    rp.scale = es;
    cudaError_t e = mp::launch_lora_reduce(rp, stream);
    if (e != cudaSuccess) return cuda_fail(c, e, "lora_reduce_kernel");
    c->eng.kernels += 1;
  }
  c->eng.lora_down += 1;
  return MP_OK;
}

// The rank-space pre-GEMM a projection launch may run as its own prologue:
// the stacked A of every live member (rtot rank rows) and the strengths.
struct Prologue {
  const CUtensorMap* tm_a = nullptr;
  int rtot = 0;
  const mp::EpilogueScale* es = nullptr;
};

// Split-K projections: per-image rows at most, and fp32 partial sums per image at most.
constexpr int kSplitRows = 1024;
constexpr size_t kSplitBytes = 32u << 20;

constexpr int kFallback = -1;  // fused launch not possible: run the pre-GEMM separately
constexpr int kSidePairs = 4;  // CTA pairs the concurrent LoRA chain needs at least

// `count` projections of one x in one launch; sts[i] (nullable) is member
// i's live stack, whose intermediate starts at column t_cols[i] of the
// scratch (row stride t_ld). With `pro`, the launch computes that
// intermediate itself (fused prologue, cooperative launch); it returns
// kFallback, having launched nothing, when that is not possible here.
// With `swi` (count 2: W1 and W3, ys[0] = h), ONE SwiGLU pair member is
// built from both: h = bf16(silu(g) * u) of their bf16 outputs.
struct SwiGluLaunch {
  const CUtensorMap* tm_bc = nullptr;  // interleaved B stack (null without live slots)
};

// With `hds`, every member is an attention-head member: ys[i] is its
// head-major output [n / 128][m][128]; norm_w[i] (nullable) turns on the
// head RMSNorm + rotary embedding for member i. With may_alloc false the
// launch grows no context buffer (the allocation-free entry point): no K split.
struct HeadsLaunch {
  const uint16_t* const* norm_w = nullptr;
  float eps = 0.0f;
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
};

int launch_projections(mp_ctx* c, const mp_weight* const* ws, void* const* ys,
                       const int64_t* ldys, const Stack* const* sts, const int* t_cols, int t_ld,
                       int count, const void* x, int64_t ldx, int m, cudaStream_t stream,
                       const Prologue* pro = nullptr, const SwiGluLaunch* swi = nullptr,
                       const HeadsLaunch* hds = nullptr, bool may_alloc = true,
                       const Prologue* sep = nullptr) {
  ProjParams p;
  int ns[mp::kMaxMembers] = {0, 0, 0, 0};
  for (int i = 0; i < count; ++i) ns[i] = ws[i]->d.n;
  // a SwiGLU pair covers 128 output features per CTA pair: as a 2N-wide member
  if (swi != nullptr) ns[0] = 2 * ws[0]->d.n;
  const int members = swi != nullptr ? 1 : count;
  // SwiGLU pairs and attention-head launches run on 256- or 512-token tiles
  // only (their kernel instantiations)
  const int mi = image_rows(c, m);
  int n_tok = 0;
  if (swi != nullptr) n_tok = std::max(mp::kMaxTok, mp::pick_ntok_pair(mi, pairs_of(ns[0])));
  if (hds != nullptr) {
    int pairs = 0;
    for (int i = 0; i < count; ++i) pairs += pairs_of(ns[i]);
    n_tok = std::max(mp::kMaxTok, mp::pick_ntok_pair(mi, pairs));
  }
  // A plain projection over few rows per image splits K across pairs: each
  // split writes fp32 partial sums (the last one after the appended LoRA K
  // tiles), lora_reduce_kernel adds them in split order and rounds to bf16.
  // The split count and the token tile come from one image's rows, at most
  // kSplitBytes of partial sums per image.
  mp::SplitChoice msplit{0, 1, 0.0};
  if (may_alloc && count == 1 && swi == nullptr && hds == nullptr && pro == nullptr && mi <= kSplitRows &&
      ns[0] % 4 == 0 && ldys[0] % 4 == 0 && reinterpret_cast<uintptr_t>(ys[0]) % 8 == 0) {
    const int base_kt = (ws[0]->d.k + mp::kBlockK - 1) / mp::kBlockK;
    const size_t per_split = static_cast<size_t>(mi) * ns[0] * sizeof(float);
    const int most = static_cast<int>(
        std::min<size_t>(mp::kMaxSplits, std::max<size_t>(1, kSplitBytes / per_split)));
    msplit = mp::choose_ksplit(mi, pairs_of(ns[0]), base_kt, ns[0], most);
    if (msplit.ksplit > 1) n_tok = msplit.n_tok;
  }
  // With `sep` (live slots whose rank-space pre-GEMM has not run yet), a
  // split-K launch runs the pre-GEMM, its reduce and the LoRA K tiles (as a
  // split of their own) on the side stream while the base splits run, on the
  // CTA pairs the base splits leave free; the final reduce adds the LoRA
  // split last. The base splits are limited so that the LoRA split's tiles
  // all fit beside them (a LoRA tile that has to wait for a base tile to end
  // would put a whole tile on the critical path). Counted on one image's
  // rows. Anything else returns kFallback having launched nothing: the caller
  // runs the pre-GEMM first and the LoRA K tiles stay in the last split.
  int side_pairs = 0;
  if (sep != nullptr) {
    if (msplit.ksplit > 1) {
      const int P = mp::resident_pairs();
      const int base_kt = (ws[0]->d.k + mp::kBlockK - 1) / mp::kBlockK;
      const size_t per_split = static_cast<size_t>(mi) * ns[0] * sizeof(float);
      const int most = static_cast<int>(
          std::min<size_t>(mp::kMaxSplits, std::max<size_t>(1, kSplitBytes / per_split)));
      // the base splits (token tile and count) that leave room for the LoRA split
      const mp::SplitChoice room =
          mp::choose_ksplit(mi, pairs_of(ns[0]), base_kt, ns[0], most, P);
      if (room.ksplit > 1) {
        const long long used = static_cast<long long>(pairs_of(ns[0])) *
                               ((mi + room.n_tok - 1) / room.n_tok) * room.ksplit;
        if (P - used >= kSidePairs) {
          msplit = room;
          n_tok = room.n_tok;
          side_pairs = static_cast<int>(P - used);
        }
      }
    }
    if (side_pairs == 0) return kFallback;
  }
  double w_bytes = 0.0;
  for (int i = 0; i < count; ++i) w_bytes += static_cast<double>(ws[i]->w_bytes);
  int rc = begin_launch(c, &p, x, ldx, ws[0]->d.k, m, ns, members, w_bytes, n_tok);
  if (rc != MP_OK) return rc;
  // prologue units are 512-token tiles: they share the member tiles' stage
  // layout and x map, so the member tiles must be 512-token tiles too
  if (pro != nullptr && (c->fuse_off || p.n_tok != mp::kMaxTileTok)) return kFallback;
  if (pro != nullptr) {
    // Fuse when the prologue units, on the pairs that run one member tile
    // fewer, lengthen the launch by less than a separate pre-GEMM would take
    // (cycle model: ~1300 / 1150 cycles per 512-token quantized / dense stage,
    // the prologue's stages dense, ~6000-8000 per tile of set-up and
    // epilogue; 1900 cycles per microsecond), modelled on one image's rows:
    // the fused prologue computes T unsplit, a separate pre-GEMM may split K,
    // so the choice must be the same for an image alone and in a batch.
    const int P = mp::resident_pairs();
    const long long n_main = static_cast<long long>(p.n_pairs) * ((mi + p.n_tok - 1) / p.n_tok);
    const long long light_pairs = P - n_main % P;
    const int base_kt = (ws[0]->d.k + mp::kBlockK - 1) / mp::kBlockK;
    int lora_kt = 0;
    for (int i = 0; i < count; ++i)
      if (sts[i] != nullptr) lora_kt = std::max(lora_kt, sts[i]->rpad / mp::kBlockK);
    if (swi != nullptr) lora_kt = t_ld / mp::kBlockK;
    const double c_stage = (ws[0]->d.bits != 0 ? 1300.0 : 1150.0) * (p.n_tok > mp::kMaxTok ? 1.0 : 0.6);
    const double t_main = (base_kt + lora_kt) * c_stage + 6000.0;
    const double t_pre = base_kt * 1150.0 + 8000.0;
    const long long n_pre = static_cast<long long>((mi + mp::kPreTok - 1) / mp::kPreTok) *
                            pairs_of(pro->rtot);
    const double heavy = static_cast<double>((n_main + P - 1) / P) * t_main;
    const double light = static_cast<double>((n_pre + light_pairs - 1) / light_pairs) * t_pre +
                         static_cast<double>(n_main / P) * t_main;
    const double fused_extra = std::max(0.0, light - heavy);
    const double separate = (mp::choose_ksplit(mi, pairs_of(pro->rtot), base_kt, pro->rtot).us + 3.0) *
                            1900.0;
    if (fused_extra >= separate) return kFallback;
  }
  if (swi != nullptr) {
    const mp_weight* w1 = ws[0];
    const mp_weight* w3 = ws[1];
    LoraTiles lt;
    if (swi->tm_bc != nullptr) {
      lt.rpad = t_ld;  // [T1 | T3]: both members' ranks
      lt.tbase = c->scratch;
      lt.t_ld = t_ld;
      lt.tm_b = swi->tm_bc;
    }
    rc = fill_member(c, &p, 0, w1->tm_w64, w1->sb, w1->sb_stride, w1->d.n, w1->d.bits, w1->d.mode,
                     ys[0], ldys[0], lt);
    if (rc != MP_OK) return rc;
    p.mem[0].swiglu = 1;
    p.mem[0].tm_w3 = w3->tm_w64;
    p.mem[0].sb3 = w3->sb;
    p.mem[0].t_col = 0;
  } else {
    for (int i = 0; i < count; ++i) {
      const mp_weight* w = ws[i];
      LoraTiles lt;
      if (sts[i] != nullptr && sts[i]->rpad > 0) {
        lt.rpad = sts[i]->rpad;
        lt.tbase = c->scratch + t_cols[i];
        lt.t_ld = t_ld;
        lt.tm_b = &sts[i]->tm_b;
      }
      rc = fill_member(c, &p, i, w->tm_w, w->sb, w->sb_stride, w->d.n, w->d.bits, w->d.mode,
                       ys[i], ldys[i], lt);
      if (rc != MP_OK) return rc;
      p.mem[i].t_col = lt.rpad > 0 ? t_cols[i] : 0;
      if (hds != nullptr) {
        mp::ProjMember& mb = p.mem[i];
        if (!encode_heads_y(&mb.tm_y, ys[i], w->d.n, m, p.n_tok))
          return fail(c, MP_ECUDA, "tensor map encode failed (head-major output)");
        mb.heads = 1;
        mb.head_norm = hds->norm_w[i] != nullptr ? 1 : 0;
        mb.norm_w = hds->norm_w[i];
        mb.norm_eps = hds->eps;
        mb.rope_cos = hds->rope_cos;
        mb.rope_sin = hds->rope_sin;
      }
    }
  }
  if (pro != nullptr) {
    p.pre_ttiles = (m + mp::kPreTok - 1) / mp::kPreTok;
    p.pre_rpairs = pairs_of(pro->rtot);
    p.n_pre = p.pre_ttiles * p.pre_rpairs;
    rc = ensure_flags(c, static_cast<size_t>(p.n_pre) * 2, stream);
    if (rc != MP_OK) return rc;
    c->epoch = c->epoch + 1 == 0 ? 1 : c->epoch + 1;
    p.flags = c->flags;
    p.epoch = c->epoch;
    if (capturing(c, stream)) {
      // a replay reuses this epoch: the flags are cleared in the graph before
      // every replay of the launch, so no flag holds it when the launch starts
      MP_CUDA(c, cudaMemsetAsync(c->flags, 0, static_cast<size_t>(p.n_pre) * 2 * sizeof(uint32_t),
                                 stream));
    }
    p.scale = *pro->es;
    mp::ProjMember& pre = p.pre;
    pre.tm_w = *pro->tm_a;
    pre.N = pro->rtot;
    pre.bits = 0;
    pre.sb = nullptr;
    pre.lora_ktiles = 0;
    if (!encode_y(&pre.tm_y, c->scratch, t_ld, pro->rtot, m, epi_box_rows(p.n_tok)))
      return fail(c, MP_ECUDA, "tensor map encode failed (rank-space intermediate)");
    cudaError_t e = mp::launch_proj_pair(p, stream);
    if (e != cudaSuccess) {
      // a cooperative launch this device refuses: nothing ran; never try again
      (void)cudaGetLastError();
      c->fuse_off = true;
      return kFallback;
    }
    c->eng.kernels += 1;
    c->eng.lora_down += 1;
  } else if (msplit.ksplit > 1) {
    const int ks = msplit.ksplit;
    const bool apart = sep != nullptr;
    const int zs = apart ? ks + 1 : ks;  // partial-sum slices: the LoRA split last
    const int n = ns[0];
    rc = ensure_buf(c, &c->part, &c->part_cap, static_cast<size_t>(zs) * m * n, stream);
    if (rc != MP_OK) return rc;
    const int k = ws[0]->d.k;
    const int base_kt = (k + mp::kBlockK - 1) / mp::kBlockK;
    p.ksplit = zs;
    p.kt_per_split = (base_kt + ks - 1) / ks;
    p.part = c->part;
    p.part_ld = n;
    if (apart) {
      // every buffer of the side chain is sized before the fork, so nothing
      // grows (or is freed) while it runs
      // pre-GEMM splits: as many as fit on the free pairs (256-token tiles)
      const int pre_max = std::max(
          1, std::min(mp::kMaxSplits,
                      side_pairs / (pairs_of(sep->rtot) * ((mi + mp::kMaxTok - 1) / mp::kMaxTok))));
      const mp::SplitChoice pre =
          mp::choose_ksplit(mi, pairs_of(sep->rtot), base_kt, sep->rtot, pre_max);
      if (pre.ksplit > 1) {
        rc = ensure_buf(c, &c->part_side, &c->part_side_cap,
                        static_cast<size_t>(pre.ksplit) * m * sep->rtot, stream);
        if (rc != MP_OK) return rc;
      }
      rc = ensure_side(c);
      if (rc != MP_OK) return rc;
      p.lora_apart = 1;
      MP_CUDA(c, cudaEventRecord(c->ev_fork, stream));
      MP_CUDA(c, cudaStreamWaitEvent(c->side, c->ev_fork, 0));
      rc = launch_lora_down(c, *sep->tm_a, sep->rtot, *sep->es, x, ldx, k, m, c->side, pre_max,
                            true);
      if (rc == MP_OK) {
        ProjParams pl = p;
        pl.z_first = ks;
        pl.z_count = 1;
        rc = run_launch(c, pl, c->side, "proj_pair_kernel (LoRA split)");
      }
      if (rc != MP_OK) {
        // joined even after a failed launch, so a capture never ends with
        // the side stream forked
        if (cudaEventRecord(c->ev_join, c->side) == cudaSuccess)
          (void)cudaStreamWaitEvent(stream, c->ev_join, 0);
        return rc;
      }
      MP_CUDA(c, cudaEventRecord(c->ev_join, c->side));
      p.z_first = 0;
      p.z_count = ks;
    }
    rc = run_launch(c, p, stream, "proj_pair_kernel (split K)");
    if (apart) {
      cudaError_t ew = cudaStreamWaitEvent(stream, c->ev_join, 0);
      if (rc != MP_OK) return rc;
      if (ew != cudaSuccess) return cuda_fail(c, ew, "cudaStreamWaitEvent (join)");
    }
    if (rc != MP_OK) return rc;
    mp::ReduceParams rp;
    std::memset(&rp, 0, sizeof(rp));  // scale.enabled = 0: the sums are stored unscaled
    rp.part = c->part;
    rp.ksplit = zs;
    rp.M = m;
    rp.R = n;
    rp.part_ld = n;
    rp.out = static_cast<uint16_t*>(ys[0]);
    rp.out_ld = static_cast<int32_t>(ldys[0]);
    cudaError_t e = mp::launch_lora_reduce(rp, stream);
    if (e != cudaSuccess) return cuda_fail(c, e, "lora_reduce_kernel (split-K projection)");
    c->eng.kernels += 1;
  } else {
    rc = run_launch(c, p, stream, "proj_pair_kernel");
    if (rc != MP_OK) return rc;
  }
  for (int i = 0; i < count; ++i)
    count_projection(c, ws[i], m, sts[i] != nullptr && sts[i]->rpad > 0 ? sts[i]->ranks : nullptr);
  return MP_OK;
}

// The stacked rank-space A over the live slots of `count` weights sharing x
// (built, or reused while no binding or live set changed), their column
// offsets col[i] in the intermediate and the strengths' epilogue scale;
// *out = nullptr and *rtot = 0 when no slot is live.
int shared_stack(mp_ctx* c, const mp_weight* const* ws, int count, cudaStream_t s,
                 mp::EpilogueScale* es, int* rtot_out, int* col, SharedStack** out) {
  std::vector<uintptr_t> key;
  std::vector<uint64_t> versions;
  int rtot = 0;
  std::memset(es, 0, sizeof(*es));
  fill_scale(c, es);
  const int k = ws[0]->d.k;
  for (int i = 0; i < count; ++i) {
    mp_weight* w = const_cast<mp_weight*>(ws[i]);
    const uint32_t mask = live_mask(c, w);
    key.push_back(reinterpret_cast<uintptr_t>(w));
    col[i] = rtot;
    if (mask != 0) {
      int rc = ensure_stack(c, w, mask, s);
      if (rc != MP_OK) return rc;
      if (!add_ranges(es, w->stack, rtot)) return fail(c, MP_EINVAL, "too many slot ranges");
      rtot += w->stack.rpad;
      versions.push_back(w->stack.version);
    } else {
      versions.push_back(0);
    }
  }
  *rtot_out = rtot;
  *out = nullptr;
  if (rtot == 0) return MP_OK;
  SharedStack& sh = c->shared[key];
  const int kp = ws[0]->kp;
  if (sh.versions != versions || sh.rtot != rtot) {
    int rc = ensure_buf(c, &sh.a, &sh.a_cap, static_cast<size_t>(rtot) * kp, s);
    if (rc != MP_OK) return rc;
    for (int i = 0; i < count; ++i) {
      const mp_weight* w = ws[i];
      if (live_mask(c, w) == 0) continue;
      MP_CUDA(c, cudaMemcpyAsync(sh.a + static_cast<size_t>(col[i]) * kp, w->stack.a,
                                 static_cast<size_t>(w->stack.rpad) * kp * 2,
                                 cudaMemcpyDeviceToDevice, s));
    }
    if (!encode_2d(&sh.tm_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, sh.a, k, rtot,
                   static_cast<uint64_t>(kp) * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B))
      return fail(c, MP_ECUDA, "tensor map encode failed (shared LoRA stack)");
    sh.versions = versions;
    sh.rtot = rtot;
  }
  *out = &sh;
  return MP_OK;
}

// The row-interleaved LoRA B stack of a SwiGLU pair: per 64-feature block b,
// rows [128b, 128b + 64) hold W1's B rows 64b.. in the columns of W1's ranks
// and rows [128b + 64, 128b + 128) W3's in the columns of W3's, zeros
// elsewhere (a 64-row W1 half and a 64-row W3 half share one MMA).
int ensure_bc(mp_ctx* c, SharedStack* sh, const mp_weight* w1, const mp_weight* w3,
              const int* col, cudaStream_t s) {
  if (sh->bc != nullptr && sh->bc_versions == sh->versions) return MP_OK;
  const int n = w1->d.n, rtot = sh->rtot;
  const int nblk = (n + 63) / 64;
  const size_t rows = static_cast<size_t>(nblk) * 128;
  int rc = ensure_buf(c, &sh->bc, &sh->bc_cap, rows * rtot, s);
  if (rc != MP_OK) return rc;
  MP_CUDA(c, cudaMemsetAsync(sh->bc, 0, rows * rtot * 2, s));
  const mp_weight* pair[2] = {w1, w3};
  for (int i = 0; i < 2; ++i) {
    const mp_weight* w = pair[i];
    if (live_mask(c, w) == 0) continue;
    const int rp = w->stack.rpad;
    for (int b = 0; b < nblk; ++b) {
      const int nr = std::min(64, n - 64 * b);
      MP_CUDA(c, cudaMemcpy2DAsync(sh->bc + (static_cast<size_t>(b) * 128 + 64 * i) * rtot + col[i],
                                   static_cast<size_t>(rtot) * 2,
                                   w->stack.b + static_cast<size_t>(b) * 64 * rp,
                                   static_cast<size_t>(rp) * 2, static_cast<size_t>(rp) * 2, nr,
                                   cudaMemcpyDeviceToDevice, s));
    }
  }
  if (!encode_2d(&sh->tm_bc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, sh->bc, rtot, rows,
                 static_cast<uint64_t>(rtot) * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B))
    return fail(c, MP_ECUDA, "tensor map encode failed (SwiGLU LoRA B stack)");
  sh->bc_versions = sh->versions;
  return MP_OK;
}

// The weight's rows with 64-row boxes, for SwiGLU pairs (64 W1 + 64 W3 rows per CTA).
int ensure_w64(mp_ctx* c, mp_weight* w) {
  if (w->has_w64) return MP_OK;
  const int n = w->d.n, k = w->d.k, bits = w->d.bits;
  bool ok;
  if (bits != 0) {
    const uint64_t row_bytes = static_cast<uint64_t>(k) * bits / 8;
    ok = encode_2d(&w->tm_w64, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->w, row_bytes, n, row_bytes,
                   64 * bits / 8, 64,
                   bits == 8 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
  } else {
    ok = encode_2d(&w->tm_w64, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, w->w, k, n,
                   static_cast<uint64_t>(w->kp) * 2, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (!ok) return fail(c, MP_ECUDA, "tensor map encode failed (64-row weight boxes)");
  w->has_w64 = true;
  return MP_OK;
}

}  // namespace

extern "C" {

const char* mp_status_string(int s) {
  switch (s) {
    case MP_OK: return "MP_OK";
    case MP_EINVAL: return "MP_EINVAL";
    case MP_ENOMEM: return "MP_ENOMEM";
    case MP_ECUDA: return "MP_ECUDA";
    case MP_ETIMEOUT: return "MP_ETIMEOUT";
    default: return "MP_UNKNOWN";
  }
}

int mp_create(int device, mp_ctx** out) {
  if (out == nullptr) return MP_EINVAL;
  *out = nullptr;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count <= 0) {
    cudaGetLastError();
    return MP_ECUDA;
  }
  if (device < 0 || device >= count) return MP_EINVAL;
  if (cudaSetDevice(device) != cudaSuccess) return MP_ECUDA;
  if (encode_fn() == nullptr) return MP_ECUDA;
  mp_ctx* c = new mp_ctx();
  c->device = device;
  for (int i = 0; i < mp::kMaxSlots; ++i) c->strength[i] = 1.0f;
  if (cudaMalloc(&c->err_word, sizeof(uint32_t)) != cudaSuccess ||
      cudaMemset(c->err_word, 0, sizeof(uint32_t)) != cudaSuccess) {
    delete c;
    return MP_ENOMEM;
  }
  *out = c;
  return MP_OK;
}

int mp_destroy(mp_ctx* c) {
  if (c == nullptr) return MP_EINVAL;
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  cudaFree(c->err_word);
  cudaFree(c->scratch);
  cudaFree(c->part);
  cudaFree(c->part_side);
  cudaFree(c->flags);
  if (c->side != nullptr) cudaStreamDestroy(c->side);
  if (c->ev_fork != nullptr) cudaEventDestroy(c->ev_fork);
  if (c->ev_join != nullptr) cudaEventDestroy(c->ev_join);
  for (void* p : c->retired) cudaFree(p);
  for (auto& kv : c->shared) {
    cudaFree(kv.second.a);
    cudaFree(kv.second.bc);
  }
  delete c;
  return MP_OK;
}

const char* mp_last_error(const mp_ctx* c) { return c == nullptr ? "null context" : c->err.c_str(); }

int mp_set_wait_limit(mp_ctx* c, uint64_t ns) {
  if (c == nullptr || ns == 0) return MP_EINVAL;
  c->wait_limit_ns = ns;
  return MP_OK;
}

int mp_sync_check(mp_ctx* c, void* stream) {
  if (c == nullptr) return MP_EINVAL;
  int rc = use_device(c);
  if (rc != MP_OK) return rc;
  MP_CUDA(c, cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  uint32_t word = 0;
  MP_CUDA(c, cudaMemcpy(&word, c->err_word, sizeof(word), cudaMemcpyDeviceToHost));
  if (word != 0) {
    MP_CUDA(c, cudaMemset(c->err_word, 0, sizeof(uint32_t)));
    return fail(c, MP_ETIMEOUT, "a kernel gave up a bounded device-side wait (word 0x%x)", word);
  }
  return MP_OK;
}

int mp_selftest_wait(mp_ctx* c, uint64_t limit_ns, void* stream) {
  if (c == nullptr) return MP_EINVAL;
  int rc = use_device(c);
  if (rc != MP_OK) return rc;
  cudaError_t e = mp::launch_wait_selftest(limit_ns, c->err_word, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(c, e, "wait_selftest_kernel");
  return MP_OK;
}

int mp_weight_upload(mp_ctx* c, const mp_weight_desc* d, const void* data, const uint16_t* scales,
                     const uint16_t* biases, mp_weight** out) {
  if (c == nullptr || d == nullptr || data == nullptr || out == nullptr) return MP_EINVAL;
  *out = nullptr;
  if (d->n <= 0 || d->k <= 0 || (d->bits != 0 && d->k % 64 != 0))
    return fail(c, MP_EINVAL,
                "weight shape [%d, %d]: n > 0 and k > 0 required, k a multiple of 64 when packed",
                d->n, d->k);
  if (d->bits != 0 && d->bits != 4 && d->bits != 8)
    return fail(c, MP_EINVAL, "bits must be 0, 4 or 8 (got %d)", d->bits);
  if (d->bits != 0) {
    if (d->group != MP_GROUP) return fail(c, MP_EINVAL, "group must be 64 (got %d)", d->group);
    if (scales == nullptr) return fail(c, MP_EINVAL, "packed weight without scales");
    if (d->mode == MP_QUANT_AFFINE && biases == nullptr)
      return fail(c, MP_EINVAL, "affine packed weight without biases");
    if (d->mode == MP_QUANT_SYMMETRIC && d->bits != 8)
      return fail(c, MP_EINVAL, "symmetric mode is 8-bit only");
    if (d->mode != MP_QUANT_AFFINE && d->mode != MP_QUANT_SYMMETRIC)
      return fail(c, MP_EINVAL, "unknown quant mode %d", d->mode);
  }
  int rc = use_device(c);
  if (rc != MP_OK) return rc;
  mp_weight* w = new mp_weight();
  w->d = *d;
  const size_t n = d->n, k = d->k;
  w->w_bytes = d->bits == 0 ? n * k * 2 : n * k * d->bits / 8;
  w->kp = (d->k + 7) / 8 * 8;
  const size_t stored = d->bits == 0 ? n * static_cast<size_t>(w->kp) * 2 : w->w_bytes;
  auto cleanup = [&](int code) {
    cudaFree(w->w);
    cudaFree(w->sb);
    delete w;
    return code;
  };
  cudaError_t e = cudaMalloc(&w->w, stored);
  if (e != cudaSuccess) return cleanup(cuda_fail(c, e, "cudaMalloc(weight)"));
  if (d->bits == 0 && w->kp != d->k) {
    e = cudaMemset(w->w, 0, stored);
    if (e == cudaSuccess)
      e = cudaMemcpy2D(w->w, static_cast<size_t>(w->kp) * 2, data, k * 2, k * 2, n,
                       cudaMemcpyDefault);
  } else {
    e = cudaMemcpy(w->w, data, stored, cudaMemcpyDefault);
  }
  if (e != cudaSuccess) return cleanup(cuda_fail(c, e, "cudaMemcpy(weight)"));
  if (d->bits != 0) {
    const int g = d->k / 64;
    w->sb_stride = (g + 3) / 4 * 4;
    std::vector<uint16_t> hs(n * g), hb(n * g, 0);
    e = cudaMemcpy(hs.data(), scales, n * g * 2, cudaMemcpyDefault);
    if (e == cudaSuccess && biases != nullptr)
      e = cudaMemcpy(hb.data(), biases, n * g * 2, cudaMemcpyDefault);
    if (e != cudaSuccess) return cleanup(cuda_fail(c, e, "cudaMemcpy(scales/biases)"));
    std::vector<uint32_t> sb(n * w->sb_stride, 0);
    for (size_t r = 0; r < n; ++r)
      for (int j = 0; j < g; ++j)
        sb[r * w->sb_stride + j] =
            static_cast<uint32_t>(hs[r * g + j]) | (static_cast<uint32_t>(hb[r * g + j]) << 16);
    e = cudaMalloc(&w->sb, sb.size() * 4);
    if (e == cudaSuccess) e = cudaMemcpy(w->sb, sb.data(), sb.size() * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cleanup(cuda_fail(c, e, "sb upload"));
    const uint64_t row_bytes = k * d->bits / 8;
    const uint32_t box_inner = 64 * d->bits / 8;
    if (!encode_2d(&w->tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->w, row_bytes, n, row_bytes,
                   box_inner, 128,
                   d->bits == 8 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B))
      return cleanup(fail(c, MP_ECUDA, "tensor map encode failed (codes)"));
  } else {
    if (!encode_2d(&w->tm_w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, w->w, k, n,
                   static_cast<uint64_t>(w->kp) * 2, 64, 128,
                   CU_TENSOR_MAP_SWIZZLE_128B))
      return cleanup(fail(c, MP_ECUDA, "tensor map encode failed (dense weight)"));
  }
  *out = w;
  return MP_OK;
}

int mp_weight_free(mp_ctx* c, mp_weight* w) {
  if (c == nullptr || w == nullptr) return MP_EINVAL;
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  // drop the shared stacks built over this weight
  for (auto it = c->shared.begin(); it != c->shared.end();) {
    const auto& key = it->first;
    if (std::find(key.begin(), key.end(), reinterpret_cast<uintptr_t>(w)) != key.end()) {
      cudaFree(it->second.a);
      cudaFree(it->second.bc);
      it = c->shared.erase(it);
    } else {
      ++it;
    }
  }
  cudaFree(w->w);
  cudaFree(w->sb);
  for (int i = 0; i < mp::kMaxSlots; ++i) {
    cudaFree(w->la[i]);
    cudaFree(w->lb[i]);
  }
  cudaFree(w->stack.a);
  cudaFree(w->stack.b);
  delete w;
  return MP_OK;
}

int mp_weight_read_codes(mp_ctx* c, const mp_weight* w, void* dst, size_t bytes) {
  if (c == nullptr || w == nullptr || dst == nullptr) return MP_EINVAL;
  if (bytes != w->w_bytes)
    return fail(c, MP_EINVAL, "read_codes: %zu bytes requested, weight holds %zu", bytes,
                w->w_bytes);
  int rc = use_device(c);
  if (rc != MP_OK) return rc;
  if (w->d.bits == 0 && w->kp != w->d.k) {
    MP_CUDA(c, cudaMemcpy2D(dst, static_cast<size_t>(w->d.k) * 2, w->w,
                            static_cast<size_t>(w->kp) * 2, static_cast<size_t>(w->d.k) * 2,
                            w->d.n, cudaMemcpyDefault));
  } else {
    MP_CUDA(c, cudaMemcpy(dst, w->w, bytes, cudaMemcpyDefault));
  }
  return MP_OK;
}

int mp_lora_bind(mp_ctx* c, mp_weight* w, int slot, const uint16_t* a, const uint16_t* b,
                 int rank) {
  if (c == nullptr || w == nullptr) return MP_EINVAL;
  if (slot < 0 || slot >= mp::kMaxSlots)
    return fail(c, MP_EINVAL, "slot %d outside [0, %d)", slot, mp::kMaxSlots);
  if (a == nullptr || b == nullptr) return fail(c, MP_EINVAL, "LoRA factor is NULL");
  if (rank <= 0 || rank > 1024) return fail(c, MP_EINVAL, "rank %d outside [1, 1024]", rank);
  int rc = use_device(c);
  if (rc != MP_OK) return rc;
  cudaDeviceSynchronize();
  cudaFree(w->la[slot]);
  cudaFree(w->lb[slot]);
  w->la[slot] = w->lb[slot] = nullptr;
  w->rank[slot] = 0;
  const size_t na = static_cast<size_t>(rank) * w->d.k, nb = static_cast<size_t>(w->d.n) * rank;
  MP_CUDA(c, cudaMalloc(&w->la[slot], na * 2));
  MP_CUDA(c, cudaMalloc(&w->lb[slot], nb * 2));
  MP_CUDA(c, cudaMemcpy(w->la[slot], a, na * 2, cudaMemcpyDefault));
  MP_CUDA(c, cudaMemcpy(w->lb[slot], b, nb * 2, cudaMemcpyDefault));
  w->rank[slot] = rank;
  w->bind_version += 1;
  c->state_version += 1;
  return MP_OK;
}

int mp_lora_unbind(mp_ctx* c, mp_weight* w, int slot) {
  if (c == nullptr || w == nullptr) return MP_EINVAL;
  if (slot < 0 || slot >= mp::kMaxSlots)
    return fail(c, MP_EINVAL, "slot %d outside [0, %d)", slot, mp::kMaxSlots);
  int rc = use_device(c);
  if (rc != MP_OK) return rc;
  cudaDeviceSynchronize();
  cudaFree(w->la[slot]);
  cudaFree(w->lb[slot]);
  w->la[slot] = w->lb[slot] = nullptr;
  w->rank[slot] = 0;
  w->bind_version += 1;
  c->state_version += 1;
  return MP_OK;
}

int mp_set_strength(mp_ctx* c, int slot, float s) {
  if (c == nullptr) return MP_EINVAL;
  if (slot < 0 || slot >= mp::kMaxSlots)
    return fail(c, MP_EINVAL, "slot %d outside [0, %d)", slot, mp::kMaxSlots);
  if (c->strength[slot] != s) c->state_version += 1;
  c->strength[slot] = s;
  return MP_OK;
}

int mp_state_version(const mp_ctx* c, uint64_t* v) {
  if (c == nullptr || v == nullptr) return MP_EINVAL;
  *v = c->state_version;
  return MP_OK;
}

int mp_get_strength(const mp_ctx* c, int slot, float* s) {
  if (c == nullptr || s == nullptr || slot < 0 || slot >= mp::kMaxSlots) return MP_EINVAL;
  *s = c->strength[slot];
  return MP_OK;
}

int mp_set_strengths_rows(mp_ctx* c, const float* s, const int32_t* row_starts, int batch) {
  if (c == nullptr) return MP_EINVAL;
  if (batch == 0) {
    if (c->n_seg != 0) c->state_version += 1;
    c->n_seg = 0;
    return MP_OK;
  }
  if (batch < 0 || batch > mp::kMaxSegments || s == nullptr || row_starts == nullptr)
    return fail(c, MP_EINVAL, "batch %d outside [0, %d] or NULL arrays", batch,
                mp::kMaxSegments);
  for (int g = 0; g < batch; ++g)
    if (row_starts[g + 1] < row_starts[g])
      return fail(c, MP_EINVAL, "row_starts must be non-decreasing");
  c->state_version += 1;
  c->n_seg = batch;
  for (int g = 0; g <= batch; ++g) c->seg_start[g] = row_starts[g];
  for (int g = 0; g < batch; ++g)
    for (int i = 0; i < mp::kMaxSlots; ++i) c->seg_scale[g][i] = s[g * mp::kMaxSlots + i];
  return MP_OK;
}

int mp_set_image_rows(mp_ctx* c, int rows) {
  if (c == nullptr) return MP_EINVAL;
  if (rows < 0) return fail(c, MP_EINVAL, "image rows %d < 0", rows);
  c->image_rows = rows;
  return MP_OK;
}

int mp_linear(mp_ctx* c, const mp_weight* wc, const void* x, int64_t ldx, void* y, int64_t ldy,
              int m, void* stream) {
  if (c == nullptr || wc == nullptr) return MP_EINVAL;
  mp_weight* w = const_cast<mp_weight*>(wc);
  int rc = check_x(c, x, ldx, w->d.k, m);
  if (rc != MP_OK) return rc;
  rc = check_y(c, y, ldy, w->d.n);
  if (rc != MP_OK) return rc;
  rc = use_device(c);
  if (rc != MP_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint32_t mask = live_mask(c, w);
  const Stack* st = nullptr;
  if (mask != 0) {
    rc = ensure_stack(c, w, mask, s);
    if (rc != MP_OK) return rc;
    st = &w->stack;
    rc = ensure_buf(c, &c->scratch, &c->scratch_cap, static_cast<size_t>(m) * st->rpad, s);
    if (rc != MP_OK) return rc;
    mp::EpilogueScale es;
    std::memset(&es, 0, sizeof(es));
    fill_scale(c, &es);
    add_ranges(&es, *st, 0);
    const mp_weight* wl[1] = {w};
    void* yl[1] = {y};
    const int64_t ll[1] = {ldy};
    const Stack* sl[1] = {st};
    const int cl[1] = {0};
    Prologue pro;
    pro.tm_a = &st->tm_a;
    pro.rtot = st->rpad;
    pro.es = &es;
    rc = launch_projections(c, wl, yl, ll, sl, cl, st->rpad, 1, x, ldx, m, s, &pro);
    if (rc != kFallback) return rc;
    rc = launch_projections(c, wl, yl, ll, sl, cl, st->rpad, 1, x, ldx, m, s, nullptr, nullptr,
                            nullptr, true, &pro);
    if (rc != kFallback) return rc;
    rc = launch_lora_down(c, st->tm_a, st->rpad, es, x, ldx, w->d.k, m, s);
    if (rc != MP_OK) return rc;
  }
  const mp_weight* wl[1] = {w};
  void* yl[1] = {y};
  const int64_t ll[1] = {ldy};
  const Stack* sl[1] = {st};
  const int cl[1] = {0};
  return launch_projections(c, wl, yl, ll, sl, cl, st != nullptr ? st->rpad : 0, 1, x, ldx, m, s);
}

int mp_linear_shared(mp_ctx* c, const mp_weight* const* ws, void* const* ys, const int64_t* ldys,
                     int count, const void* x, int64_t ldx, int m, void* stream) {
  if (c == nullptr || ws == nullptr || ys == nullptr || ldys == nullptr) return MP_EINVAL;
  if (count <= 0 || count > mp::kMaxMembers)
    return fail(c, MP_EINVAL, "count %d outside [1, %d]", count, mp::kMaxMembers);
  const int k = ws[0]->d.k;
  for (int i = 0; i < count; ++i) {
    if (ws[i] == nullptr || ws[i]->d.k != k)
      return fail(c, MP_EINVAL, "shared projections need the same k");
    int yrc = check_y(c, ys[i], ldys[i], ws[i]->d.n);
    if (yrc != MP_OK) return yrc;
  }
  int rc = check_x(c, x, ldx, k, m);
  if (rc != MP_OK) return rc;
  rc = use_device(c);
  if (rc != MP_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  mp::EpilogueScale es;
  int rtot = 0;
  int col[4] = {0, 0, 0, 0};
  SharedStack* sh = nullptr;
  rc = shared_stack(c, ws, count, s, &es, &rtot, col, &sh);
  if (rc != MP_OK) return rc;
  const Stack* sts[mp::kMaxMembers];
  for (int i = 0; i < count; ++i) sts[i] = live_mask(c, ws[i]) != 0 ? &ws[i]->stack : nullptr;
  if (rtot > 0) {
    rc = ensure_buf(c, &c->scratch, &c->scratch_cap, static_cast<size_t>(m) * rtot, s);
    if (rc != MP_OK) return rc;
    Prologue pro;
    pro.tm_a = &sh->tm_a;
    pro.rtot = rtot;
    pro.es = &es;
    rc = launch_projections(c, ws, ys, ldys, sts, col, rtot, count, x, ldx, m, s, &pro);
    if (rc != kFallback) return rc;
    rc = launch_lora_down(c, sh->tm_a, rtot, es, x, ldx, k, m, s);
    if (rc != MP_OK) return rc;
  }
  return launch_projections(c, ws, ys, ldys, sts, col, rtot, count, x, ldx, m, s);
}

int mp_linear_heads(mp_ctx* c, const mp_weight* const* ws, void* const* ys, int count,
                    const void* x, int64_t ldx, int m, const uint16_t* const* norm_w, float eps,
                    const float* rope_cos, const float* rope_sin, void* stream) {
  if (c == nullptr || ws == nullptr || ys == nullptr) return MP_EINVAL;
  if (count <= 0 || count > mp::kMaxMembers)
    return fail(c, MP_EINVAL, "count %d outside [1, %d]", count, mp::kMaxMembers);
  const int k = ws[0] != nullptr ? ws[0]->d.k : 0;
  bool any_norm = false;
  for (int i = 0; i < count; ++i) {
    if (ws[i] == nullptr || ws[i]->d.k != k)
      return fail(c, MP_EINVAL, "head projections need the same k");
    if (ws[i]->d.n % mp::kHeadDim != 0)
      return fail(c, MP_EINVAL, "n = %d is not a whole number of %d-wide heads", ws[i]->d.n,
                  mp::kHeadDim);
    if (ys[i] == nullptr || reinterpret_cast<uintptr_t>(ys[i]) % 16 != 0)
      return fail(c, MP_EINVAL, "head-major output %d is NULL or not 16-byte aligned", i);
    if (norm_w != nullptr && norm_w[i] != nullptr) {
      if (reinterpret_cast<uintptr_t>(norm_w[i]) % 16 != 0)
        return fail(c, MP_EINVAL, "norm gain %d must be 16-byte aligned", i);
      any_norm = true;
    }
  }
  if (any_norm) {
    if (rope_cos == nullptr || rope_sin == nullptr ||
        reinterpret_cast<uintptr_t>(rope_cos) % 16 != 0 ||
        reinterpret_cast<uintptr_t>(rope_sin) % 16 != 0)
      return fail(c, MP_EINVAL, "the normed heads need 16-byte aligned rotary tables");
    if (!(eps > 0.0f)) return fail(c, MP_EINVAL, "eps must be positive");
  }
  int rc = check_x(c, x, ldx, k, m);
  if (rc != MP_OK) return rc;
  rc = use_device(c);
  if (rc != MP_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint16_t* nw[mp::kMaxMembers] = {nullptr, nullptr, nullptr, nullptr};
  for (int i = 0; i < count; ++i) nw[i] = norm_w != nullptr ? norm_w[i] : nullptr;
  HeadsLaunch hds;
  hds.norm_w = nw;
  hds.eps = eps;
  hds.rope_cos = rope_cos;
  hds.rope_sin = rope_sin;
  int64_t lds[mp::kMaxMembers];
  for (int i = 0; i < count; ++i) lds[i] = ws[i]->d.n;  // token-major stride, unused by the 3-D map
  mp::EpilogueScale es;
  int rtot = 0;
  int col[4] = {0, 0, 0, 0};
  SharedStack* sh = nullptr;
  rc = shared_stack(c, ws, count, s, &es, &rtot, col, &sh);
  if (rc != MP_OK) return rc;
  const Stack* sts[mp::kMaxMembers] = {nullptr, nullptr, nullptr, nullptr};
  for (int i = 0; i < count; ++i) sts[i] = live_mask(c, ws[i]) != 0 ? &ws[i]->stack : nullptr;
  if (rtot > 0) {
    rc = ensure_buf(c, &c->scratch, &c->scratch_cap, static_cast<size_t>(m) * rtot, s);
    if (rc != MP_OK) return rc;
    Prologue pro;
    pro.tm_a = &sh->tm_a;
    pro.rtot = rtot;
    pro.es = &es;
    rc = launch_projections(c, ws, ys, lds, sts, col, rtot, count, x, ldx, m, s, &pro, nullptr,
                            &hds);
    if (rc != kFallback) return rc;
    rc = launch_lora_down(c, sh->tm_a, rtot, es, x, ldx, k, m, s);
    if (rc != MP_OK) return rc;
  }
  return launch_projections(c, ws, ys, lds, sts, col, rtot, count, x, ldx, m, s, nullptr, nullptr,
                            &hds);
}

int mp_attention(mp_ctx* c, const void* q, const void* k, const void* v, int s, int nh,
                 int64_t head_stride, float scale, void* o, int64_t ldo, void* stream) {
  if (c == nullptr) return MP_EINVAL;
  if (s <= 0 || nh <= 0) return fail(c, MP_EINVAL, "s and nh must be positive (%d, %d)", s, nh);
  if (!(scale > 0.0f)) return fail(c, MP_EINVAL, "scale must be positive");
  for (const void* t : {q, k, v, static_cast<const void*>(o)})
    if (t == nullptr || reinterpret_cast<uintptr_t>(t) % 16 != 0)
      return fail(c, MP_EINVAL, "q, k, v and o must be non-NULL and 16-byte aligned");
  if (ldo < static_cast<int64_t>(nh) * mp::kHeadDim || ldo % 8 != 0)
    return fail(c, MP_EINVAL, "ldo must be >= 128 * nh and a multiple of 8 (got %lld)",
                static_cast<long long>(ldo));
  if (head_stride == 0) head_stride = static_cast<int64_t>(s) * mp::kHeadDim;
  if (head_stride < static_cast<int64_t>(s) * mp::kHeadDim || head_stride % 8 != 0)
    return fail(c, MP_EINVAL, "head_stride must be >= 128 * s and a multiple of 8 (got %lld)",
                static_cast<long long>(head_stride));
  int rc = use_device(c);
  if (rc != MP_OK) return rc;
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(c, MP_ECUDA, "cuTensorMapEncodeTiled unavailable");
  mp::AttnParams p;
  std::memset(&p, 0, sizeof(p));
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(mp::kHeadDim), static_cast<cuuint64_t>(s),
                              static_cast<cuuint64_t>(nh)};
  const cuuint64_t strides[2] = {mp::kHeadDim * 2, static_cast<cuuint64_t>(head_stride) * 2};
  // q and v: boxes of 64 dims x 128 rows; k: 64 dims x 64 keys (each CTA of a
  // pair loads half of a 128-key step)
  const cuuint32_t boxes[3][3] = {{64, 128, 1}, {64, 64, 1}, {64, 128, 1}};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUtensorMap* maps[3] = {&p.tm_q, &p.tm_k, &p.tm_v};
  const void* srcs[3] = {q, k, v};
  for (int i = 0; i < 3; ++i)
    if (fn(maps[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(srcs[i]), dims, strides,
           boxes[i], estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return fail(c, MP_ECUDA, "tensor map encode failed (attention operand %d)", i);
  p.o = static_cast<uint16_t*>(o);
  p.ldo = ldo;
  p.S = s;
  p.NH = nh;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.wait_limit_ns = c->wait_limit_ns;
  p.err = c->err_word;
  cudaError_t e = mp::launch_attention(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(c, e, "attn_kernel");
  c->eng.kernels += 1;
  return MP_OK;
}

int mp_rms_residual(mp_ctx* c, void* x, int64_t ldx, const void* o, int64_t ldo,
                    const void* o_gain, const void* gate, void* nrm, int64_t ldn,
                    const void* nrm_gain, int h, int m, float eps, void* stream) {
  if (c == nullptr) return MP_EINVAL;
  if (h <= 0 || h % 8 != 0 || h > mp::kNormMaxH)
    return fail(c, MP_EINVAL, "h = %d must be a positive multiple of 8, at most %d", h,
                mp::kNormMaxH);
  if (m <= 0) return fail(c, MP_EINVAL, "m must be positive (got %d)", m);
  if (!(eps > 0.0f)) return fail(c, MP_EINVAL, "eps must be positive");
  auto row_ok = [&](const void* ptr, int64_t ld) {
    return ptr != nullptr && reinterpret_cast<uintptr_t>(ptr) % 16 == 0 && ld >= h && ld % 8 == 0;
  };
  auto vec_ok = [&](const void* ptr) {
    return ptr != nullptr && reinterpret_cast<uintptr_t>(ptr) % 16 == 0;
  };
  if (!row_ok(x, ldx)) return fail(c, MP_EINVAL, "x: NULL, not 16-byte aligned or bad ldx");
  if (o != nullptr && (!row_ok(o, ldo) || !vec_ok(o_gain)))
    return fail(c, MP_EINVAL, "o: bad rows or o_gain NULL / not 16-byte aligned");
  if (o == nullptr && gate != nullptr) return fail(c, MP_EINVAL, "gate without o");
  if (nrm != nullptr && (!row_ok(nrm, ldn) || !vec_ok(nrm_gain)))
    return fail(c, MP_EINVAL, "nrm: bad rows or nrm_gain NULL / not 16-byte aligned");
  if (o == nullptr && nrm == nullptr) return fail(c, MP_EINVAL, "nothing to compute");
  int rc = use_device(c);
  if (rc != MP_OK) return rc;
  mp::RmsResidualParams p;
  p.x = static_cast<uint16_t*>(x);
  p.ldx = ldx;
  p.o = static_cast<const uint16_t*>(o);
  p.ldo = ldo;
  p.o_gain = static_cast<const uint16_t*>(o_gain);
  p.gate = static_cast<const uint16_t*>(gate);
  p.nrm = static_cast<uint16_t*>(nrm);
  p.ldn = ldn;
  p.nrm_gain = static_cast<const uint16_t*>(nrm_gain);
  p.M = m;
  p.H = h;
  p.eps = eps;
  cudaError_t e = mp::launch_rms_residual(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(c, e, "rms_residual_kernel");
  c->eng.kernels += 1;
  return MP_OK;
}

int mp_linear_swiglu(mp_ctx* c, const mp_weight* w1, const mp_weight* w3, const void* x,
                     int64_t ldx, void* h, int64_t ldh, int m, void* stream) {
  if (c == nullptr || w1 == nullptr || w3 == nullptr) return MP_EINVAL;
  if (w1->d.n != w3->d.n || w1->d.k != w3->d.k || w1->d.bits != w3->d.bits ||
      w1->d.mode != w3->d.mode)
    return fail(c, MP_EINVAL, "SwiGLU gate and up weights need the same shape and format");
  const int n = w1->d.n, k = w1->d.k;
  int rc = check_x(c, x, ldx, k, m);
  if (rc != MP_OK) return rc;
  rc = check_y(c, h, ldh, n);
  if (rc != MP_OK) return rc;
  rc = use_device(c);
  if (rc != MP_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const mp_weight* ws[2] = {w1, w3};
  for (const mp_weight* w : ws) {
    rc = ensure_w64(c, const_cast<mp_weight*>(w));
    if (rc != MP_OK) return rc;
  }
  mp::EpilogueScale es;
  int rtot = 0;
  int col[4] = {0, 0, 0, 0};
  SharedStack* sh = nullptr;
  rc = shared_stack(c, ws, 2, s, &es, &rtot, col, &sh);
  if (rc != MP_OK) return rc;
  void* ys[2] = {h, nullptr};
  const int64_t lds[2] = {ldh, ldh};
  const Stack* sts[mp::kMaxMembers] = {nullptr, nullptr, nullptr, nullptr};
  for (int i = 0; i < 2; ++i) sts[i] = live_mask(c, ws[i]) != 0 ? &ws[i]->stack : nullptr;
  SwiGluLaunch swi;
  if (rtot > 0) {
    rc = ensure_bc(c, sh, w1, w3, col, s);
    if (rc != MP_OK) return rc;
    swi.tm_bc = &sh->tm_bc;
    rc = ensure_buf(c, &c->scratch, &c->scratch_cap, static_cast<size_t>(m) * rtot, s);
    if (rc != MP_OK) return rc;
    Prologue pro;
    pro.tm_a = &sh->tm_a;
    pro.rtot = rtot;
    pro.es = &es;
    rc = launch_projections(c, ws, ys, lds, sts, col, rtot, 2, x, ldx, m, s, &pro, &swi);
    if (rc != kFallback) return rc;
    rc = launch_lora_down(c, sh->tm_a, rtot, es, x, ldx, k, m, s);
    if (rc != MP_OK) return rc;
  }
  return launch_projections(c, ws, ys, lds, sts, col, rtot, 2, x, ldx, m, s, nullptr, &swi);
}

int mp_modulation_create(mp_ctx* c, int n_blocks, const mp_weight* const* ada,
                         const uint16_t* const* ada_bias, const uint16_t* const* an1,
                         const uint16_t* const* fn1, mp_modset** out) {
  if (c == nullptr || ada == nullptr || ada_bias == nullptr || out == nullptr) return MP_EINVAL;
  *out = nullptr;
  if (n_blocks <= 0) return fail(c, MP_EINVAL, "n_blocks must be positive");
  const mp_weight_desc& d0 = ada[0]->d;
  if (d0.n % 4 != 0) return fail(c, MP_EINVAL, "modulation n must be 4*H");
  for (int i = 0; i < n_blocks; ++i) {
    const mp_weight_desc& d = ada[i]->d;
    if (d.n != d0.n || d.k != d0.k || d.bits != d0.bits || d.mode != d0.mode)
      return fail(c, MP_EINVAL, "modulation weights must share shape and format");
    if (ada_bias[i] == nullptr) return fail(c, MP_EINVAL, "modulation bias %d is NULL", i);
    if (d.k % 8 != 0) return fail(c, MP_EINVAL, "modulation k must be a multiple of 8");
  }
  int rc = use_device(c);
  if (rc != MP_OK) return rc;
  mp_modset* set = new mp_modset();
  set->n_blocks = n_blocks;
  set->n = d0.n;
  set->k = d0.k;
  set->bits = d0.bits;
  set->mode = d0.mode;
  set->sb_stride = ada[0]->sb_stride;
  const int H = d0.n / 4;
  std::vector<mp::ModBlock> hb(n_blocks);
  auto copy_vec = [&](const uint16_t* src, size_t elems, const uint16_t** dst) -> int {
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, elems * 2);
    if (e == cudaSuccess) e = cudaMemcpy(p, src, elems * 2, cudaMemcpyDefault);
    if (e != cudaSuccess) return cuda_fail(c, e, "modulation vector upload");
    set->owned.push_back(p);
    *dst = static_cast<const uint16_t*>(p);
    return MP_OK;
  };
  for (int i = 0; i < n_blocks; ++i) {
    hb[i].w = static_cast<const uint8_t*>(ada[i]->w);
    hb[i].sb = ada[i]->sb;
    hb[i].an1 = nullptr;
    hb[i].fn1 = nullptr;
    int r = copy_vec(ada_bias[i], d0.n, &hb[i].bias);
    if (r == MP_OK && an1 != nullptr && an1[i] != nullptr) r = copy_vec(an1[i], H, &hb[i].an1);
    if (r == MP_OK && fn1 != nullptr && fn1[i] != nullptr) r = copy_vec(fn1[i], H, &hb[i].fn1);
    if (r != MP_OK) {
      for (void* p : set->owned) cudaFree(p);
      delete set;
      return r;
    }
  }
  // the lane-per-row kernel (K a multiple of 256, N of 128) streams 32 rows x
  // 128 bytes per step with one TMA; other shapes take the generic kernel
  const bool lane_maps = d0.k % 256 == 0 && d0.n % 128 == 0;
  std::vector<CUtensorMap> hm(lane_maps ? n_blocks : 0);
  for (int i = 0; i < static_cast<int>(hm.size()); ++i) {
    const mp_weight* w = ada[i];
    bool ok;
    if (d0.bits != 0) {
      const uint64_t row_bytes = static_cast<uint64_t>(d0.k) * d0.bits / 8;
      ok = encode_2d(&hm[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, w->w, row_bytes, d0.n, row_bytes, 128,
                     32, CU_TENSOR_MAP_SWIZZLE_128B);
    } else {
      ok = encode_2d(&hm[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, w->w, d0.k, d0.n,
                     static_cast<uint64_t>(w->kp) * 2, 64, 32, CU_TENSOR_MAP_SWIZZLE_128B);
    }
    if (!ok) {
      for (void* p : set->owned) cudaFree(p);
      delete set;
      return fail(c, MP_ECUDA, "tensor map encode failed (modulation weights)");
    }
  }
  cudaError_t e = cudaMalloc(&set->dev_blocks, sizeof(mp::ModBlock) * n_blocks);
  if (e == cudaSuccess)
    e = cudaMemcpy(set->dev_blocks, hb.data(), sizeof(mp::ModBlock) * n_blocks,
                   cudaMemcpyHostToDevice);
  if (e == cudaSuccess && lane_maps) e = cudaMalloc(&set->dev_maps, sizeof(CUtensorMap) * n_blocks);
  if (e == cudaSuccess && lane_maps)
    e = cudaMemcpy(set->dev_maps, hm.data(), sizeof(CUtensorMap) * n_blocks, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    for (void* p : set->owned) cudaFree(p);
    cudaFree(set->dev_blocks);
    cudaFree(set->dev_maps);
    delete set;
    return cuda_fail(c, e, "modulation table upload");
  }
  *out = set;
  return MP_OK;
}

int mp_modulation_free(mp_ctx* c, mp_modset* set) {
  if (c == nullptr || set == nullptr) return MP_EINVAL;
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  for (void* p : set->owned) cudaFree(p);
  cudaFree(set->dev_blocks);
  cudaFree(set->dev_maps);
  delete set;
  return MP_OK;
}

int mp_modulation_all(mp_ctx* c, const mp_modset* set, const void* temb, int m, void* mods,
                      void* nw1, void* nw3, void* stream) {
  if (c == nullptr || set == nullptr || temb == nullptr || mods == nullptr) return MP_EINVAL;
  if (m <= 0 || m > mp::kModMaxBatch)
    return fail(c, MP_EINVAL, "modulation m %d outside [1, %d]", m, mp::kModMaxBatch);
  int rc = use_device(c);
  if (rc != MP_OK) return rc;
  mp::ModParams p;
  std::memset(&p, 0, sizeof(p));
  p.blocks = set->dev_blocks;
  p.n_blocks = set->n_blocks;
  p.N = set->n;
  p.K = set->k;
  p.H = set->n / 4;
  p.bits = set->bits;
  const bool sym = set->bits == 8 && set->mode == MP_QUANT_SYMMETRIC;
  p.code_xor = sym ? 0x80808080u : 0u;
  p.code_magic = sym ? 8388736.0f : 8388608.0f;
  p.sb_stride = set->sb_stride;
  p.m_stride = m;
  p.maps = set->dev_maps;
  p.err = c->err_word;
  p.wait_limit_ns = c->wait_limit_ns;
  // launches of at most a few tokens (8 on the tensor-core path); every
  // token's row is computed the same way whichever launch holds it
  const int per_launch = mp::mod_tokens_per_launch(set->n, set->k, set->n_blocks);
  for (int m0 = 0; m0 < m; m0 += per_launch) {
    p.M = std::min(per_launch, m - m0);
    p.temb = static_cast<const uint16_t*>(temb) + static_cast<size_t>(m0) * set->k;
    p.mods = static_cast<uint16_t*>(mods) + static_cast<size_t>(m0) * set->n;
    p.nw1 = nw1 != nullptr ? static_cast<uint16_t*>(nw1) + static_cast<size_t>(m0) * p.H : nullptr;
    p.nw3 = nw3 != nullptr ? static_cast<uint16_t*>(nw3) + static_cast<size_t>(m0) * p.H : nullptr;
    cudaError_t e = mp::launch_mod(p, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(c, e, "mod_kernel");
    c->eng.kernels += 1;
  }
  c->eng.modulation += 1;
  const double wbytes = set->bits == 0 ? 2.0 * set->n * set->k : set->n * set->k * set->bits / 8.0;
  c->eng.flops += 2.0 * m * set->n * static_cast<double>(set->k) * set->n_blocks;
  c->eng.bytes += set->n_blocks * (wbytes + (set->bits ? set->n * (set->k / 64) * 4.0 : 0.0) +
                                   2.0 * set->n * (1 + m));
  return MP_OK;
}

int mp_engagement_get(const mp_ctx* c, mp_engagement* out) {
  if (c == nullptr || out == nullptr) return MP_EINVAL;
  *out = c->eng;
  return MP_OK;
}

int mp_engagement_reset(mp_ctx* c) {
  if (c == nullptr) return MP_EINVAL;
  c->eng = mp_engagement{};
  return MP_OK;
}

}  // extern "C"

// ---- allocation-free entry point ---------------------------------------------
//
// Some callers cannot call cudaMalloc: a host whose memory planner owns every
// device allocation up front (the plugin's host hands out pooled buffers and
// budgets device memory per session), and latency-critical serving loops in
// which an allocation or a free could synchronize the device. For them,
// mp_linear_lora_static runs one adapter's fused projection with its
// rank-space intermediate held in a fixed, file-scope device array instead of
// context scratch. Every GPU that loads this library holds the array (4 MiB)
// until the process exits.

// Elements (bf16) of the shared rank-space scratch: m * roundup(rank, 64) must fit.
#define MP_STATIC_RANK_SCRATCH_ELEMS (static_cast<size_t>(2) << 20)

static __device__ __align__(256) uint16_t g_static_rank_scratch[MP_STATIC_RANK_SCRATCH_ELEMS];

namespace {

// Device address of g_static_rank_scratch, looked up once per device with that
// device current (host code only has a host-side stand-in for the symbol).
// Atomic, so two host threads making their first call on the same device at
// once both store the same value without a data race.
std::atomic<uint16_t*> g_static_rank_scratch_dev[64] = {};

int static_rank_scratch(mp_ctx* c, uint16_t** out) {
  if (c->device < 0 || c->device >= 64) return fail(c, MP_EINVAL, "device index out of range");
  uint16_t* p = g_static_rank_scratch_dev[c->device].load(std::memory_order_acquire);
  if (p == nullptr) {
    void* sym = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&sym, g_static_rank_scratch);
    if (e != cudaSuccess) return cuda_fail(c, e, "cudaGetSymbolAddress(g_static_rank_scratch)");
    p = static_cast<uint16_t*>(sym);
    g_static_rank_scratch_dev[c->device].store(p, std::memory_order_release);
  }
  *out = p;
  return MP_OK;
}

}  // namespace

extern "C" int mp_linear_lora_static(mp_ctx* c, const mp_weight* w, const void* x, int64_t ldx,
                                     const uint16_t* a, const uint16_t* b, int rank,
                                     float strength, void* y, int64_t ldy, int m, void* stream) {
  if (c == nullptr || w == nullptr) return MP_EINVAL;
  int rc = check_x(c, x, ldx, w->d.k, m);
  if (rc != MP_OK) return rc;
  rc = check_y(c, y, ldy, w->d.n);
  if (rc != MP_OK) return rc;
  if (a == nullptr || b == nullptr) return fail(c, MP_EINVAL, "LoRA factor is NULL");
  if (rank <= 0 || rank > 256 || rank % 8 != 0)
    return fail(c, MP_EINVAL, "rank %d: must be a multiple of 8 in [8, 256]", rank);
  if (reinterpret_cast<uintptr_t>(a) % 16 != 0 || reinterpret_cast<uintptr_t>(b) % 16 != 0)
    return fail(c, MP_EINVAL, "LoRA factors must be 16-byte aligned device memory");
  if (w->d.k % 8 != 0) return fail(c, MP_EINVAL, "k must be a multiple of 8 here");
  const int rpad = (rank + 63) / 64 * 64;
  if (static_cast<size_t>(m) * rpad > MP_STATIC_RANK_SCRATCH_ELEMS)
    return fail(c, MP_EINVAL,
                "m * roundup(rank, 64) = %lld exceeds the static scratch of %zu elements",
                static_cast<long long>(m) * rpad, static_cast<size_t>(MP_STATIC_RANK_SCRATCH_ELEMS));
  rc = use_device(c);
  if (rc != MP_OK) return rc;
  uint16_t* scratch = nullptr;
  rc = static_rank_scratch(c, &scratch);
  if (rc != MP_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int n = w->d.n, k = w->d.k;
  const mp_weight* wl[1] = {w};
  void* yl[1] = {y};
  const int64_t ll[1] = {ldy};
  if (strength == 0.0f) {
    const Stack* none[1] = {nullptr};
    const int cols[1] = {0};
    return launch_projections(c, wl, yl, ll, none, cols, 0, 1, x, ldx, m, s, nullptr, nullptr,
                              nullptr, /*may_alloc=*/false);
  }

  // Rank-space pre-GEMM into the static array: all rpad columns are written
  // (rows of `a` past `rank` read as zeros), so nothing left from an earlier
  // call survives into this one.
  CUtensorMap tm_a;
  if (!encode_2d(&tm_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a, k, rank,
                 static_cast<uint64_t>(k) * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B))
    return fail(c, MP_ECUDA, "tensor map encode failed (static LoRA A)");
  // the token tile the separate pre-GEMM would take, without a K split (its
  // fp32 partial sums would need memory this entry point does not allocate)
  const mp::SplitChoice sc =
      mp::choose_ksplit(m, pairs_of(rpad), (k + mp::kBlockK - 1) / mp::kBlockK, rpad, 1);
  ProjParams p;
  rc = begin_launch(c, &p, x, ldx, k, m, &rpad, 1, 2.0 * rpad * k, sc.n_tok);
  if (rc != MP_OK) return rc;
  p.scale.enabled = 1;
  p.scale.n_seg = 1;
  p.scale.seg_start[0] = 0;
  p.scale.seg_start[1] = INT_MAX;
  p.scale.seg_scale[0][0] = strength;
  p.scale.n_ranges = 1;
  p.scale.range_start[0] = 0;
  p.scale.range_start[1] = rank;
  p.scale.range_slot[0] = 0;
  rc = fill_member(c, &p, 0, tm_a, nullptr, 0, rpad, 0, 0, scratch, rpad, LoraTiles{});
  if (rc != MP_OK) return rc;
  rc = run_launch(c, p, s, "proj_pair_kernel (static rank-space pre-GEMM)");
  if (rc != MP_OK) return rc;
  c->eng.lora_down += 1;

  // The fused projection with the adapter appended as extra K tiles; `b`'s
  // columns past `rank` read as zeros.
  CUtensorMap tm_bl;
  if (!encode_2d(&tm_bl, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, b, rank, n,
                 static_cast<uint64_t>(rank) * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B))
    return fail(c, MP_ECUDA, "tensor map encode failed (static LoRA B)");
  ProjParams q;
  rc = begin_launch(c, &q, x, ldx, k, m, &n, 1, static_cast<double>(w->w_bytes));
  if (rc != MP_OK) return rc;
  LoraTiles lt;
  lt.rpad = rpad;
  lt.tbase = scratch;
  lt.t_ld = rpad;
  lt.tm_b = &tm_bl;
  rc = fill_member(c, &q, 0, w->tm_w, w->sb, w->sb_stride, n, w->d.bits, w->d.mode, y, ldy, lt);
  if (rc != MP_OK) return rc;
  rc = run_launch(c, q, s, "proj_pair_kernel (static LoRA projection)");
  if (rc != MP_OK) return rc;
  int ranks[mp::kMaxSlots] = {rank};
  count_projection(c, w, m, ranks);
  return MP_OK;
}
