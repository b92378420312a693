// Paged GQA/MQA decode attention for sm_100a (one query token per sequence),
// with the step's KV append fused in.
//
// Replaces the decode step of qwen model.rs:390-416: the new K/V row is
// stored at position seq_len-1 (the paged form of the Tensor::cat at
// model.rs:390-392), then q head h attends over every key of KV head
// h / n_rep (model.rs:398-408) with scores q.k * scale (model.rs:298, 413),
// softmax over all keys including the reference's all-zero first row
// (model.rs:207-220, flag MTN_ATTN_PHANTOM_ZERO_SLOT) and output P.V
// (model.rs:416).  One query token sees every key, so generate_causal_mask
// (model.rs:542-555) masks nothing here.
//
// Design.  The step is HBM-bound (each K/V byte is read once) but at
// n_rep = 7 the arithmetic is 3.5 FMA per byte, more than the CUDA cores
// issue at HBM speed, so both contractions run on the tensor cores with the
// query heads of one KV head as the narrow N dimension:
//   S^T[128 tokens][16] = K_tile[128][D] . Q^T            (tcgen05, M = 128, N = 16)
//   O^T[D][16]         += V_tile^T[D][128] . P^T[128][16] (tcgen05, M = 64 | 128, N = 16)
// Persistent grid: SMs x CTAs-per-SM CTAs.  The (sequence, kv head)
// segments are cut into 128-token tiles, laid end to end, and every CTA
// takes an equal contiguous range of tiles (computed on the device from
// seq_lens), so the producer streams TMA loads across segment boundaries
// without bubbles.  10 warps per CTA:
//   warps 0-3  softmax: TMEM lane = token; online softmax in the exp2 domain
//              against a CTA-wide reference max that moves only when a tile
//              exceeds it by 2^8 (lazy rescale), P^T (bf16) to shared memory;
//              at a segment's end they hand its row sums and maxima to the
//              epilogue warps and go on with the next segment's tiles.
//   warp 4     producer: per segment the Q^T operand, per tile one TMA box
//              per page per 64-wide head-dim block straight from the block
//              table into a 3-stage ring (at head_dim 256: a 6-slot ring of
//              head-dim halves, 1.5 tiles), and the fused KV append.
//   warp 5     MMA issuer (one thread); S^T double-buffered in TMEM so the
//              next tile's QK^T overlaps this tile's softmax; O^T
//              double-buffered per segment so an epilogue overlaps the next
//              segment.
//   warps 6-9  segment epilogues: O^T out of TMEM once the segment's last
//              P V is done, normalised outputs or partials, merge tickets
//              and the merges.
// A segment cut by CTA boundaries leaves (m, l, O) partials in per-CTA
// workspace slots.  After its last tile each CTA takes a ticket for the (at
// most two) segments it only holds part of; the last CTA to arrive merges
// that segment's pieces in CTA order (no spinning, nothing stalls the tile
// pipeline), so results do not depend on scheduling.  Every wait is bounded.
#include <algorithm>
#include <cfloat>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "tc.cuh"
#include "tmaps.hpp"

// Scratch of mtn_paged_decode_noalloc: a file-scope device array, so the
// library image itself reserves it on every device that loads it.
static __device__ __align__(256) unsigned char mtn_noalloc_decode_scratch[8u << 20];

namespace mtn {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
// Work plan of a decode launch, made on the host (int32 words):
//   [0] kPlanMagic  [1] participating CTAs  [2] grid it was made for  [3] tiles U
//   [4 + 8 c + k] CTA c: t0, n_local, start sequence, tiles (one kv head's) of
//                 the sequences before it, its valid length, its first page index
//   [4 + 8 grid + c] CTA boundaries, c = 0 .. grid (participating CTAs .. grid: U)
constexpr int32_t kPlanMagic = 0x504e544d;  // "MTNP"
constexpr int kPlanEntry = 8;
constexpr int kTile = 128;    // tokens per tile = MMA1 M = TMEM lanes
constexpr int kThreads = 320;  // 10 warps: softmax 0-3, producer 4, MMA 5, epilogue 6-9
constexpr int kEpiWarp0 = 6;
constexpr int kN = 16;        // query heads per KV head, padded (MMA N)
// P is exponentiated against a reference max that moves only when a tile's
// max exceeds it by more than 2^8, so P <= 256 and O^T is rarely rescaled.
constexpr float kRescaleLog2 = 8.0f;
// Page id of a box position past its sequence's last page (never a valid id).
constexpr int kPastEnd = -0x40000000;

struct DecodeParams {
  int64_t num_pages;
  int64_t row_k;  // pool-view row of (layer K, page 0, head 0, token 0)
  int64_t row_v;
  __nv_bfloat16* pool;  // for the fused append (generic stores)
  int hkv;
  int ps;
  int hq;
  int n_seqs;
  const void* q;
  void* o;
  int q_f32;
  int o_f32;
  const void* k_new;  // optional [n_seqs][hkv][D]
  const void* v_new;
  int new_f32;
  const int32_t* kv_indptr;
  const int32_t* kv_indices;
  const int32_t* seq_lens;
  float qscale;  // scale * log2(e)
  int phantom;
  float* ws_o;           // [ctas][2][16][D]   partial O of split segments
  float* ws_ml;          // [ctas][2][16][2]   partial (m, l)
  unsigned int* ws_cnt;  // [n_seqs][hkv]      arrival tickets (left at zero)
  int* err;
  const int32_t* plan;   // host-made work plan (mtn_paged_decode_plan) or null
  float* lse;            // [n_seqs][hq] log2-domain log-sum-exp of each row, or null
  int oob_row;           // a pool-view row past the tensor (its boxes read as zeros), or -1
};

template <int D>
struct DCfg {
  static constexpr int kDB = D / 64;                       // 64-wide head-dim blocks
  // D = 256: K and V of a tile are staged as head-dim halves (32 KB items,
  // 4 per tile) in a 6-slot ring, so 1.5 tiles are in flight; otherwise
  // kStages whole-tile K+V stages.  kStages is also how many tiles ahead the
  // producer fetches page ids (1 for D = 256: measured faster than 3 there).
  static constexpr bool kHalf = D == 256;
  static constexpr int kStages = D == 256 ? 1 : 3;
  static constexpr int kRingSlots = 6;
  static constexpr int kHalfBytes = kTile * 128 * 2;       // 128 tokens x two 64-column blocks
  static constexpr int kCtasPerSm = D == 64 ? 2 : 1;
  static constexpr int kQBytes = kN * D * 2;               // Q^T operand: 16 rows x D
  static constexpr int kKVBytes = kTile * D * 2;           // one of K or V per stage
  static constexpr int kPBytes = kN * kTile * 2;           // P^T operand: 16 rows x 128 tokens
  // Small state first, then the 1 KiB-aligned operand area.
  static constexpr int kOffBar = 0;                        // 28 mbarriers
  static constexpr int kOffMisc = kOffBar + 28 * 8;        // tmem base, abort, last flag, start info
  // [2][4][16] tile maxima; per O^T buffer [2][4][16] warp row sums and [2][16] reference maxima
  static constexpr int kOffRed = kOffMisc + 64;
  static constexpr int kOffScan = kOffRed + (2 * 4 * kN + 2 * 4 * kN + 2 * kN) * 4;  // [10] warp totals
  static constexpr int kOffPend = kOffScan + (kThreads / 32) * 8;                   // [2] int4 deferred merges
  static constexpr int kSmallBytes = kOffPend + 32 + 16;
  static constexpr int kOffQ = 0;                          // [2] relative to the aligned operand area
  static constexpr int kOffK = kOffQ + 2 * kQBytes;
  static constexpr int kOffV = kHalf ? kOffK : kOffK + kStages * kKVBytes;
  static constexpr int kOffP = kHalf ? kOffK + kRingSlots * kHalfBytes : kOffV + kStages * kKVBytes;
  static constexpr int kBigBytes = kOffP + 2 * kPBytes;  // P^T double-buffered
  static constexpr int kSmem = kSmallBytes + 1023 + kBigBytes;
  static constexpr int kMO = D == 64 ? 64 : 128;           // MMA2 M
  static constexpr int kTmemS = 0;                          // [2] x 16 columns
  static constexpr int kTmemO = 32;                         // [2] x 32 columns
  static constexpr int kTmemCols = 128;
  static_assert(kOffK % 1024 == 0 && kOffV % 1024 == 0 && kOffP % 1024 == 0, "swizzle atoms need 1 KiB alignment");
};

enum Bar {
  kKVFull0 = 0,   // [6] stage (or ring slot) loaded
  kKVEmpty0 = 6,  // [6] stage (or ring slot) consumed
  kSFull0 = 12,   // [2]
  kPFull0 = 14,   // [2] P^T buffer i&1 written (softmax -> MMA)
  kODone0 = 16,   // [2] P V of tile i done: P^T buffer i&1 free, O^T current
  kQFull0 = 18,   // [2]
  kQEmpty0 = 20,  // [2]
  kOFree0 = 22,   // [2] O^T buffer read out by the epilogue (and its sums slot free)
  kEFull0 = 24,   // [2] softmax state of the segment in O^T buffer b handed to the epilogue
  kOSeg0 = 26,    // [2] last P V of the segment in O^T buffer b done
  kNumBars = 28
};
static_assert(kNumBars * 8 <= DCfg<64>::kOffMisc, "mbarrier area");
static_assert(DCfg<64>::kOffPend % 16 == 0 && DCfg<128>::kOffPend % 16 == 0, "int4 alignment");

// A segment's arrival ticket: one atomic add at gpu scope with acquire and
// release semantics.  Release: the partials this CTA's threads wrote before
// the named barrier that precedes the call are visible to whoever acquires
// a later ticket; acquire: this CTA's reads after the next barrier see every
// partial released by earlier tickets (the merge reads them with ld.cg).
__device__ __forceinline__ unsigned int ticket_add(unsigned int* cnt) {
  unsigned int r;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(r) : "l"(cnt) : "memory");
  return r;
}

// Final normalisation of one output element: o/l with the phantom key folded in.
__device__ __forceinline__ float finalize(float o, float l, float m, int phantom) {
  if (phantom) {
    const float mf = fmaxf(m, 0.0f);  // m == -inf (no real keys) gives mf = 0
    const float a = (m == -INFINITY) ? 0.0f : exp2f(m - mf);
    l = l * a + exp2f(-mf);
    o = o * a;
  }
  return l > 0.0f ? o / l : 0.0f;
}

__device__ __forceinline__ void store_out(const DecodeParams& p, int64_t idx, float v) {
  if (p.o_f32) static_cast<float*>(p.o)[idx] = v;
  else static_cast<__nv_bfloat16*>(p.o)[idx] = __float2bfloat16_rn(v);
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  tc::tmem_ld_wait();
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}

// Valid length of sequence s, clamped to its block table (an out-of-range
// value records kDevErrBadSeqLen, from CTA 0 only).
__device__ __forceinline__ int seq_len_of(const DecodeParams& p, int s) {
  const int ntab = p.kv_indptr[s + 1] - p.kv_indptr[s];
  const int len = p.seq_lens[s];
  if (len < 0 || len > ntab * p.ps) {
    if (blockIdx.x == 0) record_error(p.err, kDevErrBadSeqLen, s);
    return min(max(len, 0), ntab * p.ps);
  }
  return len;
}

// Walks a CTA's tiles in order: (sequence s, kv head g, tile j of T).
struct Walker {
  int s, g, j, T, len, pbeg;
  int64_t pre;  // tiles (in units of one kv head) of the sequences before s

  __device__ void load(const DecodeParams& p) {
    len = seq_len_of(p, s);
    T = (len + kTile - 1) / kTile;
    pbeg = p.kv_indptr[s];
  }
  // Start at global tile t0 of sequence s0 whose metadata is already known.
  __device__ void start(const DecodeParams& p, int s0, int64_t pre0, int64_t t0, int len0, int pbeg0) {
    s = s0;
    pre = pre0;
    len = len0;
    T = (len + kTile - 1) / kTile;
    pbeg = pbeg0;
    const int64_t off = t0 - pre * p.hkv;
    g = static_cast<int>(off / T);
    j = static_cast<int>(off - static_cast<int64_t>(g) * T);
  }
  // Only called while tiles remain, so a non-empty sequence follows.
  __device__ void next(const DecodeParams& p) {
    if (++j < T) return;
    j = 0;
    if (++g < p.hkv) return;
    g = 0;
    do {
      pre += T;
      ++s;
      load(p);
    } while (T == 0 && s + 1 < p.n_seqs);
  }
  __device__ int64_t seg_start(const DecodeParams& p) const { return pre * p.hkv + static_cast<int64_t>(g) * T; }
};

// CTA c's first tile and the CTA whose range holds global tile x: from the
// plan's boundary table (bnd, in shared memory) when there is one, else the
// equal split c * U / C.
__device__ __forceinline__ int64_t tile_begin(const int32_t* bnd, int64_t c, int64_t U, int64_t C) {
  return bnd ? bnd[c] : c * U / C;
}
__device__ __forceinline__ int64_t cta_of(const int32_t* bnd, int64_t x, int64_t U, int64_t C) {
  if (!bnd) return min(C - 1, ((x + 1) * C - 1) / U);
  int64_t lo = 0, hi = C - 1;  // the last c with bnd[c] <= x
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (bnd[mid] <= x) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// PREC (MTN_ATTN_SPLIT_BF16): Q and P enter the tensor cores as bf16 hi +
// lo pairs, hi = bf16(x) and lo = bf16(x - hi), so each product carries
// about 16 mantissa bits of its f32 operand instead of 8.  N = 16 holds at
// most 8 query heads, so the lo rows ride in rows 8..15 of the same Q^T and
// P^T operands: S^T columns h and h + 8 (and O^T columns h and h + 8) are
// the hi and lo products of head h, summed in f32 -- no extra MMA.
// LSE: also store each row's log-sum-exp in p.lse (the shared-prefix decode);
// a separate instantiation, so the plain decode's code is untouched.
template <int D, int NREP, bool PREC, bool LSE = false>
__global__ void __launch_bounds__(kThreads, DCfg<D>::kCtasPerSm)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tm_kv, const __grid_constant__ CUtensorMap tm_q,
                        const __grid_constant__ DecodeParams p) {
  using C = DCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw + C::kOffBar);
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(smem_raw + C::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem_raw + C::kOffMisc + 4);
  int* start_s = reinterpret_cast<int*>(smem_raw + C::kOffMisc + 12);
  int64_t* start_pre = reinterpret_cast<int64_t*>(smem_raw + C::kOffMisc + 16);
  int* start_len = reinterpret_cast<int*>(smem_raw + C::kOffMisc + 32);
  int* start_pbeg = reinterpret_cast<int*>(smem_raw + C::kOffMisc + 36);
  float* red_max = reinterpret_cast<float*>(smem_raw + C::kOffRed);  // [2][4][16]
  float* red_l = red_max + 2 * 4 * kN;                               // [2][4][16]
  float* red_m = red_l + 2 * 4 * kN;                                 // [2][16]
  int64_t* scan = reinterpret_cast<int64_t*>(smem_raw + C::kOffScan);  // [6]
  int4* pend = reinterpret_cast<int4*>(smem_raw + C::kOffPend);        // [2] (segment, ca, cb, wa)
  volatile int* last_flag = reinterpret_cast<volatile int*>(smem_raw + C::kOffPend + 32);  // [2]
  uint8_t* big = smem_raw + C::kSmallBytes;
  big += (1024 - (smem_u32(big) & 1023)) & 1023;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tid = threadIdx.x;
  const int64_t cta = blockIdx.x;

  // Programmatic dependent launch: the next kernel of the stream (the next
  // decode launch, the next layer's or step's) may start its own prologue on
  // SMs this launch frees; it waits for this grid to finish (griddepcontrol
  // .wait below) before it reads or writes anything this grid touches.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // TMEM first.  Measured with %globaltimer on B200: the second CTA of an SM
  // started only once the first had allocated TMEM and given up its
  // allocation permit (2.5 us late when that came after the metadata scan,
  // 0.7 us when it comes first).
  if (warp == 0) {
    tc::tmem_alloc(tmem_base_s, C::kTmemCols);
    tc::tmem_relinquish();
    tc::fence_before_sync();
  }

  // ------------------------------------------------------------ work split
  // Each thread owns a contiguous chunk of sequences (the scan below, and the
  // outputs of sequences without tiles).
  const int chunk = (p.n_seqs + kThreads - 1) / kThreads;
  const int sb = min(p.n_seqs, tid * chunk), se = min(p.n_seqs, sb + chunk);
  if (tid == 0) {
    for (int i = 0; i < kNumBars; ++i)
      mbar_init(&bars[i], (i == kPFull0 || i == kPFull0 + 1 || i == kEFull0 || i == kEFull0 + 1) ? 4
                          : (i == kOFree0 || i == kOFree0 + 1)                              ? 128
                                                                                            : 1);
    *abort_flag = 0;
    *start_s = -1;
    fence_barrier_init();
  }
  int64_t U = 0, ctas = 0, t0 = 0;
  int n_local = 0;
  const int32_t* bnd = nullptr;  // the plan's CTA boundaries (shared memory) when there is a plan
  if (p.plan != nullptr) {
    // Host-made plan: this CTA's range and start, and every CTA's first
    // tile, in one round of independent loads.
    const int32_t* pl = p.plan;
    int32_t* bnd_s = reinterpret_cast<int32_t*>(big + C::kBigBytes);
    for (int i = tid; i <= static_cast<int>(gridDim.x); i += kThreads) bnd_s[i] = pl[4 + kPlanEntry * gridDim.x + i];
    const int32_t* e = pl + 4 + kPlanEntry * cta;
    const bool plan_ok = pl[0] == kPlanMagic && pl[2] == static_cast<int32_t>(gridDim.x) && pl[1] >= 0 &&
                         pl[1] <= static_cast<int32_t>(gridDim.x);
    if (plan_ok) {
      ctas = pl[1];
      U = pl[3];
      if (cta < ctas) {
        t0 = e[0];
        n_local = e[1];
        if (tid == 0) {
          *start_s = e[2];
          *start_pre = e[3];
          *start_len = e[4];
          *start_pbeg = e[5];
        }
      }
    } else if (tid == 0 && cta == 0) {
      record_error(p.err, kDevErrBadPlan, pl[0] == kPlanMagic ? pl[2] : -1);
    }
    bnd = bnd_s;
  } else {
    // Tiles per sequence (for one kv head), prefix-summed over the CTA.
    int64_t mine = 0;
    int len_first = 0;  // metadata of this thread's first sequence, kept for the start search
    for (int s = sb; s < se; ++s) {
      const int len = seq_len_of(p, s);
      const int T = (len + kTile - 1) / kTile;
      if (s == sb) len_first = len;
      mine += T;
    }
    int64_t incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) scan[warp] = incl;
    __syncthreads();
    int64_t before = incl - mine;
    for (int w = 0; w < warp; ++w) before += scan[w];
    int64_t total_seq_tiles = 0;
    for (int w = 0; w < kThreads / 32; ++w) total_seq_tiles += scan[w];
    U = total_seq_tiles * p.hkv;
    // With fewer tiles than CTAs only the first U CTAs take part, so every
    // participating CTA owns at least one tile and a segment's pieces are
    // exactly the CTAs cta_of(first tile) .. cta_of(last tile).
    ctas = min(static_cast<int64_t>(gridDim.x), U);
    t0 = cta < ctas ? tile_begin(nullptr, cta, U, ctas) : 0;
    n_local = static_cast<int>(cta < ctas ? tile_begin(nullptr, cta + 1, U, ctas) - t0 : 0);
    if (n_local > 0 && t0 >= before * p.hkv && t0 < (before + mine) * p.hkv) {
      int64_t pre = before;
      for (int s = sb; s < se; ++s) {
        const int len = (s == sb) ? len_first : seq_len_of(p, s);
        const int T = (len + kTile - 1) / kTile;
        if (t0 < (pre + T) * p.hkv) {
          *start_s = s;
          *start_pre = pre;
          *start_len = len;
          *start_pbeg = p.kv_indptr[s];
          break;
        }
        pre += T;
      }
    }
  }
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_base_s;
  // Up to here the CTA read only the batch metadata (seq_lens, kv_indptr),
  // which no decode launch writes; it may have started while the previous
  // kernel of the stream was still running (see launch_dependents above).
  // Each role waits for that kernel (griddepcontrol.wait) before it reads
  // q, k_new/v_new or K/V pages, or writes o, the pool or the workspace:
  // the producer only after fetching its first tiles' page ids, which are
  // metadata too.  (A kernel that does not allow early launch has finished
  // before this grid starts: then the wait returns at once.)
  auto grid_wait = [] { asm volatile("griddepcontrol.wait;" ::: "memory"); };
  // Sequences without tiles: nobody else writes their output (phantom-only
  // or empty softmax).  Run by every thread after its wait.
  auto empty_outputs = [&] {
    for (int s = sb; s < se; ++s) {
      if (s % static_cast<int64_t>(gridDim.x) != cta) continue;
      const int len = seq_len_of(p, s);
      if ((len + kTile - 1) / kTile == 0) {
        const float z = finalize(0.0f, 0.0f, -INFINITY, p.phantom);
        for (int e = 0; e < p.hq * D; ++e) store_out(p, static_cast<int64_t>(s) * p.hq * D + e, z);
        if constexpr (LSE)
          for (int h = 0; h < p.hq; ++h) p.lse[static_cast<int64_t>(s) * p.hq + h] = row_lse(p.phantom, -INFINITY, 0.0f);
      }
    }
  };
  // Uniform over the CTA.  The bad start cannot happen for consistent metadata.
  const bool bad_start = n_local > 0 && (*start_s < 0 || *start_s >= p.n_seqs);
  if (n_local == 0 || bad_start) {
    grid_wait();
    empty_outputs();
    if (bad_start && tid == 0) record_error(p.err, kDevErrBadSeqLen, -1);
    if (warp == 0) tc::tmem_dealloc(tmem, C::kTmemCols);
    return;
  }

  uint8_t* p_s = big + C::kOffP;
  if (warp < 4 || warp == 5) {
    // The zeroed P^T operand (rows >= NREP stay zero) for the MMA and
    // softmax roles; the producer starts loading meanwhile.
    const int tid160 = warp == 5 ? 128 + lane : tid;
    uint4* pz = reinterpret_cast<uint4*>(p_s);
    for (int e = tid160; e < 2 * C::kPBytes / 16; e += 160) pz[e] = make_uint4(0u, 0u, 0u, 0u);
    grid_wait();
    empty_outputs();
    fence_proxy_async_shared();
    tc::named_sync(2, 160);
  }
  const int s0 = *start_s;
  const int64_t pre0 = *start_pre;
  const int len0 = *start_len, pbeg0 = *start_pbeg;
  const int tile_pages = kTile / p.ps;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tc::prefetch_tmap(&tm_kv);
      if (!p.q_f32) tc::prefetch_tmap(&tm_q);
    }
    Walker w;   // the tile whose loads are issued
    w.start(p, s0, pre0, t0, len0, pbeg0);
    Walker wp = w;  // the tile whose page ids are fetched, kStages tiles ahead
    int qcnt = 0;
    // Per stage slot: this lane's page id of the slot's tile and, when that
    // tile ends its segment, the page and offset of this step's K/V row for
    // the fused append plus the row itself.  Fetched kStages tiles ahead, so
    // the first kStages tiles are issued back to back and later fetches
    // overlap the wait for a free stage; the ids are checked only when used,
    // so no fetch waits for its own load.
    int pg[C::kStages], apg[C::kStages], apos[C::kStages];
    int64_t asrc[C::kStages];  // element offset of the appended row in k_new / v_new
    uint4 ak[C::kStages], av[C::kStages];
    auto load_rows = [&](int64_t src, uint4& ak_o, uint4& av_o) {
      if (lane >= D / 8) return;
      src += lane * 8;
      if (p.new_f32) {
        const float* kf = static_cast<const float*>(p.k_new) + src;
        const float* vf = static_cast<const float*>(p.v_new) + src;
        const float4 k0 = *reinterpret_cast<const float4*>(kf), k1 = *reinterpret_cast<const float4*>(kf + 4);
        const float4 v0 = *reinterpret_cast<const float4*>(vf), v1 = *reinterpret_cast<const float4*>(vf + 4);
        ak_o = make_uint4(f2_to_bf2(k0.x, k0.y), f2_to_bf2(k0.z, k0.w), f2_to_bf2(k1.x, k1.y), f2_to_bf2(k1.z, k1.w));
        av_o = make_uint4(f2_to_bf2(v0.x, v0.y), f2_to_bf2(v0.z, v0.w), f2_to_bf2(v1.x, v1.y), f2_to_bf2(v1.z, v1.w));
      } else {
        ak_o = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.k_new) + src);
        av_o = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.v_new) + src);
      }
    };
    // Page ids of wp's tile and, when that tile ends its segment, the page
    // and offset of this step's row; the row itself (k_new / v_new, which the
    // previous kernel may have written) only when `rows` is set.
    auto fetch = [&](int& pg_o, int& apg_o, int& apos_o, int64_t& asrc_o, uint4& ak_o, uint4& av_o, bool rows) {
      const int npg = (wp.len + p.ps - 1) / p.ps;
      pg_o = 0;
      // Box positions past the sequence's last page take no page id: their
      // boxes are loaded from p.oob_row, which the TMA unit fills with zeros
      // without reading memory (kPastEnd); the softmax masks those tokens.
      if (lane < tile_pages) {
        const int pi = wp.j * tile_pages + lane;
        pg_o = (pi >= npg && p.oob_row >= 0) ? kPastEnd : p.kv_indices[wp.pbeg + min(pi, npg - 1)];
      }
      apos_o = -1;  // no append
      apg_o = 0;
      ak_o = make_uint4(0u, 0u, 0u, 0u);
      av_o = ak_o;
      if (p.k_new != nullptr && wp.j == wp.T - 1) {
        const int pos = wp.len - 1;
        apos_o = pos % p.ps;
        apg_o = p.kv_indices[wp.pbeg + pos / p.ps];
        asrc_o = (static_cast<int64_t>(wp.s) * p.hkv + wp.g) * D;
        if (rows) load_rows(asrc_o, ak_o, av_o);
      }
    };
#pragma unroll
    for (int k = 0; k < C::kStages; ++k) {
      if (k < n_local) fetch(pg[k], apg[k], apos[k], asrc[k], ak[k], av[k], false);
      if (k + 1 < n_local) wp.next(p);
    }
    grid_wait();
#pragma unroll
    for (int k = 0; k < C::kStages; ++k)
      if (k < n_local && apos[k] >= 0) load_rows(asrc[k], ak[k], av[k]);
    bool run = true;
    // Stage slot st of round i0 is tile i0 + st.  At two CTAs per SM (head_dim
    // 64) the loop body is kept rolled (the smaller code measured faster
    // there) and the ring registers rotate by one slot per tile, so tile i's
    // values are always slot 0 and the fetch fills the last slot: constant
    // indices keep the ring in registers (indexed by st it lived in local
    // memory; rotating measured 2-4 % faster at 64-1024 sequences).  At
    // head_dim >= 128 the body is unrolled and slot st holds tile i0 + st
    // (config 5: 0.80 vs 0.74 of HBM for the rolled loop).
    constexpr bool kRot = C::kCtasPerSm > 1;
    for (int i0 = 0; run && i0 < n_local; i0 += C::kStages) {
#pragma unroll (kRot ? 1 : C::kStages)
      for (int st = 0; st < C::kStages; ++st) {
        const int i = i0 + st;
        const int rs = kRot ? 0 : st;  // ring slot of tile i
        if (!run || i >= n_local) break;
        const bool first = (i == 0) || w.j == 0;
        if (first) {
          const int qb = qcnt & 1;
          if (qcnt >= 2) {
            bool ok = true;
            if (lane == 0) ok = tc::wait_bounded(&bars[kQEmpty0 + qb], ((qcnt >> 1) - 1) & 1, abort_flag, p.err, 11);
            if (!__shfl_sync(0xffffffffu, ok, 0)) {
              run = false;
              break;
            }
          }
          uint8_t* q_s = big + C::kOffQ + qb * C::kQBytes;
          const int qrow = w.s * p.hq + w.g * NREP;
          if (!p.q_f32) {
            // Rows past NREP belong to other heads (or lie past the end and
            // read as zero): their S^T columns are never used.
            if (lane == 0) {
              mbar_arrive_expect_tx(&bars[kQFull0 + qb], C::kQBytes);
#pragma unroll
              for (int b = 0; b < C::kDB; ++b)
                tc::tma_load_3d(q_s + b * (kN * 128), &tm_q, b * 64, 0, qrow, &bars[kQFull0 + qb]);
            }
          } else {
            for (int e = lane; e < NREP * (D / 8); e += 32) {
              const int r = e / (D / 8), c = e - r * (D / 8);
              const float* src = static_cast<const float*>(p.q) + (static_cast<int64_t>(qrow) + r) * D + c * 8;
              const float4 a = *reinterpret_cast<const float4*>(src);
              const float4 b2 = *reinterpret_cast<const float4*>(src + 4);
              const uint4 hi =
                  make_uint4(f2_to_bf2(a.x, a.y), f2_to_bf2(a.z, a.w), f2_to_bf2(b2.x, b2.y), f2_to_bf2(b2.z, b2.w));
              *reinterpret_cast<uint4*>(q_s + (c >> 3) * (kN * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4)) = hi;
              if constexpr (PREC) {
                // row r + 8: the bf16 remainders (r + 8 has the same swizzle phase as r)
                const uint4 lo = make_uint4(bf2_residual(hi.x, a.x, a.y), bf2_residual(hi.y, a.z, a.w),
                                            bf2_residual(hi.z, b2.x, b2.y), bf2_residual(hi.w, b2.z, b2.w));
                *reinterpret_cast<uint4*>(q_s + (c >> 3) * (kN * 128) + (r + 8) * 128 + (((c & 7) ^ (r & 7)) << 4)) =
                    lo;
              }
            }
            fence_proxy_async_shared();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&bars[kQFull0 + qb]);
          }
          ++qcnt;
        }
        if (!C::kHalf && i >= C::kStages) {
          bool ok = true;
          if (lane == 0)
            ok = tc::wait_bounded(&bars[kKVEmpty0 + st], ((i / C::kStages) - 1) & 1, abort_flag, p.err, 10);
          if (!__shfl_sync(0xffffffffu, ok, 0)) {
            run = false;
            break;
          }
        }
        if (apos[rs] >= 0) {
          // Fused KV append: store this step's row at position len-1, then
          // order it before the async-proxy (TMA) read of the same page.
          if (apg[rs] < 0 || apg[rs] >= p.num_pages) {
            if (lane == 0) record_error(p.err, kDevErrBadPage, w.s);
          } else if (lane < D / 8) {
            const int64_t arow = (static_cast<int64_t>(apg[rs]) * p.hkv + w.g) * p.ps + apos[rs];
            *reinterpret_cast<uint4*>(p.pool + (p.row_k + arow) * D + lane * 8) = ak[rs];
            *reinterpret_cast<uint4*>(p.pool + (p.row_v + arow) * D + lane * 8) = av[rs];
            asm volatile("fence.proxy.async.global;" ::: "memory");
          }
          __syncwarp();
        }
        if constexpr (C::kHalf) {
          // Items 4i..4i+3 of the ring: K blocks 0-1, K blocks 2-3, V blocks
          // 0-1, V blocks 2-3; item n sits in slot n % 6, refilled once the
          // MMA that read item n - 6 is done.
          int64_t page = lane < tile_pages ? pg[rs] : 0;
          const bool past = page == kPastEnd;
          if (lane < tile_pages && !past && (page < 0 || page >= p.num_pages)) {
            record_error(p.err, kDevErrBadPage, w.s);
            page = 0;  // reload a valid page instead (masked)
          }
          const int64_t rk = past ? p.oob_row : p.row_k + (page * p.hkv + w.g) * p.ps;
          const int64_t rv = past ? p.oob_row : p.row_v + (page * p.hkv + w.g) * p.ps;
          for (int hh = 0; hh < 4; ++hh) {
            const int n = 4 * i + hh;
            const int slot = n % C::kRingSlots;
            bool ok = true;
            if (lane == 0 && n >= C::kRingSlots)
              ok = tc::wait_bounded(&bars[kKVEmpty0 + slot], ((n / C::kRingSlots) - 1) & 1, abort_flag, p.err, 12);
            if (!__shfl_sync(0xffffffffu, ok, 0)) {
              run = false;
              break;
            }
            if (lane == 0) mbar_arrive_expect_tx(&bars[kKVFull0 + slot], C::kHalfBytes);
            __syncwarp();
            if (lane < tile_pages) {
              uint8_t* dst = big + C::kOffK + slot * C::kHalfBytes + lane * p.ps * 128;
              const int row = static_cast<int>(hh < 2 ? rk : rv);
#pragma unroll
              for (int bb = 0; bb < 2; ++bb)
                tc::tma_load_2d(dst + bb * kTile * 128, &tm_kv, ((hh & 1) * 2 + bb) * 64, row,
                                &bars[kKVFull0 + slot]);
            }
          }
          if (!run) break;
        } else {
        if (lane == 0) mbar_arrive_expect_tx(&bars[kKVFull0 + st], 2 * C::kKVBytes);
        __syncwarp();
        if (lane < tile_pages) {
          int64_t page = pg[rs];
          const bool past = page == kPastEnd;
          if (!past && (page < 0 || page >= p.num_pages)) {
            record_error(p.err, kDevErrBadPage, w.s);
            page = 0;  // reload a valid page instead (masked)
          }
          const int64_t rk = past ? p.oob_row : p.row_k + (page * p.hkv + w.g) * p.ps;
          const int64_t rv = past ? p.oob_row : p.row_v + (page * p.hkv + w.g) * p.ps;
          uint8_t* kst = big + C::kOffK + st * C::kKVBytes;
          uint8_t* vst = big + C::kOffV + st * C::kKVBytes;
#pragma unroll
          for (int b = 0; b < C::kDB; ++b) {
            const int off = b * kTile * 128 + lane * p.ps * 128;
            tc::tma_load_2d(kst + off, &tm_kv, b * 64, static_cast<int>(rk), &bars[kKVFull0 + st]);
            tc::tma_load_2d(vst + off, &tm_kv, b * 64, static_cast<int>(rv), &bars[kKVFull0 + st]);
          }
        }
        }
        if constexpr (kRot) {
#pragma unroll
          for (int k = 0; k + 1 < C::kStages; ++k) {
            pg[k] = pg[k + 1];
            apg[k] = apg[k + 1];
            apos[k] = apos[k + 1];
            asrc[k] = asrc[k + 1];
            ak[k] = ak[k + 1];
            av[k] = av[k + 1];
          }
        }
        if (i + C::kStages < n_local) {
          const int fs = kRot ? C::kStages - 1 : st;  // wp is at tile i + kStages
          fetch(pg[fs], apg[fs], apos[fs], asrc[fs], ak[fs], av[fs], true);
          if (i + C::kStages + 1 < n_local) wp.next(p);
        }
        if (i + 1 < n_local) w.next(p);
      }
    }
    empty_outputs();  // off the first loads' path
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = tc::idesc_bf16(kTile, kN, false, false);
      constexpr uint32_t idO = tc::idesc_bf16(C::kMO, kN, false, true);
      Walker wsw, wo;  // wsw: tiles whose S^T is issued; wo: tiles whose O^T is issued
      wsw.start(p, s0, pre0, t0, len0, pbeg0);
      wo.start(p, s0, pre0, t0, len0, pbeg0);
      int q_seg = -1;  // segment counter of the S^T issue
      int o_seg = -1;  // segment counter of the O^T issue
      // Operand descriptors of stage 0 / buffer 0 at k = 0; the others add
      // their byte offset >> 4 to the start-address field (shared addresses
      // stay below 256 KB, so the 14-bit field never carries).
      const uint64_t dK = tc::sdesc_sw128(smem_u32(big + C::kOffK), 16, 1024);
      const uint64_t dQ = tc::sdesc_sw128(smem_u32(big + C::kOffQ), 16, 1024);
      const uint64_t dV = tc::sdesc_sw128(smem_u32(big + C::kOffV), kTile * 128, 1024);
      const uint64_t dP = tc::sdesc_sw128(smem_u32(p_s), 16, 1024);
      // S^T(i) = K_i Q^T into S buffer i&1: both operands K-major; 16-wide
      // k steps walk 32 bytes inside a 128-byte swizzle row, then the next block.
      auto issue_s = [&](int i) -> bool {
        const bool first = (i == 0) || wsw.j == 0;
        const bool last = (i == n_local - 1) || wsw.j == wsw.T - 1;
        if (first) {
          ++q_seg;
          if (!tc::wait_bounded(&bars[kQFull0 + (q_seg & 1)], (q_seg >> 1) & 1, abort_flag, p.err, 22)) return false;
        }
        const uint64_t b0 = dQ + (((q_seg & 1) * C::kQBytes) >> 4);
        if constexpr (C::kHalf) {
          // K halves: ring items 4i (blocks 0-1) and 4i+1 (blocks 2-3).
          const int s0 = (4 * i) % C::kRingSlots, s1 = (4 * i + 1) % C::kRingSlots;
          if (!tc::wait_bounded(&bars[kKVFull0 + s0], ((4 * i) / C::kRingSlots) & 1, abort_flag, p.err, 24) ||
              !tc::wait_bounded(&bars[kKVFull0 + s1], ((4 * i + 1) / C::kRingSlots) & 1, abort_flag, p.err, 25))
            return false;
          tc::fence_after_sync();
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const int slot = (k >> 3) ? s1 : s0;
            tc::mma_bf16(tmem + C::kTmemS + (i & 1) * kN,
                         dK + ((slot * C::kHalfBytes + ((k >> 2) & 1) * kTile * 128 + (k & 3) * 32) >> 4),
                         b0 + (((k >> 2) * kN * 128 + (k & 3) * 32) >> 4), idS, k > 0 ? 1u : 0u);
          }
          tc::mma_commit(&bars[kSFull0 + (i & 1)]);
          tc::mma_commit(&bars[kKVEmpty0 + s0]);
          tc::mma_commit(&bars[kKVEmpty0 + s1]);
        } else {
        const int st = i % C::kStages;
        if (!tc::wait_bounded(&bars[kKVFull0 + st], (i / C::kStages) & 1, abort_flag, p.err, 20)) return false;
        tc::fence_after_sync();
        const uint64_t a0 = dK + ((st * C::kKVBytes) >> 4);
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          tc::mma_bf16(tmem + C::kTmemS + (i & 1) * kN, a0 + (((k >> 2) * kTile * 128 + (k & 3) * 32) >> 4),
                       b0 + (((k >> 2) * kN * 128 + (k & 3) * 32) >> 4), idS, k > 0 ? 1u : 0u);
        tc::mma_commit(&bars[kSFull0 + (i & 1)]);
        }
        if (last) tc::mma_commit(&bars[kQEmpty0 + (q_seg & 1)]);
        if (i + 1 < n_local) wsw.next(p);
        return true;
      };
      // Can S^T(j) be issued without waiting?  (wsw is positioned at tile j.)
      auto s_ready = [&](int j) -> bool {
        const bool first = (j == 0) || wsw.j == 0;
        if (first && !mbar_test_wait(&bars[kQFull0 + ((q_seg + 1) & 1)], ((q_seg + 1) >> 1) & 1)) return false;
        if constexpr (C::kHalf)
          return mbar_test_wait(&bars[kKVFull0 + (4 * j) % C::kRingSlots], ((4 * j) / C::kRingSlots) & 1) &&
                 mbar_test_wait(&bars[kKVFull0 + (4 * j + 1) % C::kRingSlots], ((4 * j + 1) / C::kRingSlots) & 1);
        return mbar_test_wait(&bars[kKVFull0 + j % C::kStages], (j / C::kStages) & 1);
      };
      bool ok = true;
      int next_s = 0;  // next tile whose S^T is not issued yet
      for (int i = 0; ok && i < n_local; ++i) {
        // Issue S^T(i) if it is not out yet (waiting for its K/V), then wait
        // for P^T(i), issuing S^T(i+1) as soon as its K/V land (its S buffer
        // was released by the softmax of tile i-1, whose P^T was waited on in
        // the previous iteration).  One call site keeps the loop's code small.
        {
          uint64_t* pf = &bars[kPFull0 + (i & 1)];
          const uint32_t par = (i >> 1) & 1;
          uint64_t t_start = 0;
          for (uint32_t it = 0;; ++it) {
            if (next_s <= i || (next_s == i + 1 && next_s < n_local && s_ready(next_s))) {
              ok = issue_s(next_s);
              ++next_s;
              if (!ok) break;
              continue;
            }
            if (mbar_test_wait(pf, par)) break;
            // Back off between polls: this warp shares a scheduler with a
            // softmax warp, which a tight spin would starve.
            __nanosleep(32);
            if ((it & 255u) == 0) {
              const uint64_t now = tc::global_timer_ns();
              if (it == 0) t_start = now;
              if (*abort_flag) {
                ok = false;
                break;
              }
              if (now - t_start > 1000000000ull) {
                record_error(p.err, kDevErrTimeout, 21);
                *abort_flag = 1;
                ok = false;
                break;
              }
            }
          }
          if (!ok) break;
        }
        const bool first = (i == 0) || wo.j == 0;
        const bool last_o = (i == n_local - 1) || wo.j == wo.T - 1;
        if (first) {
          ++o_seg;
          if (o_seg >= 2 &&
              !tc::wait_bounded(&bars[kOFree0 + (o_seg & 1)], ((o_seg >> 1) - 1) & 1, abort_flag, p.err, 23))
            break;
        }
        const uint64_t b0 = dP + (((i & 1) * C::kPBytes) >> 4);
        const uint32_t o_col = C::kTmemO + (o_seg & 1) * 32;
        if constexpr (C::kHalf) {
          // V halves: ring items 4i+2 (head dims 0-127) and 4i+3 (128-255),
          // one M = 128 block of O^T each.
          const int s2 = (4 * i + 2) % C::kRingSlots, s3 = (4 * i + 3) % C::kRingSlots;
          if (!tc::wait_bounded(&bars[kKVFull0 + s2], ((4 * i + 2) / C::kRingSlots) & 1, abort_flag, p.err, 26) ||
              !tc::wait_bounded(&bars[kKVFull0 + s3], ((4 * i + 3) / C::kRingSlots) & 1, abort_flag, p.err, 27))
            break;
          tc::fence_after_sync();
#pragma unroll
          for (int k = 0; k < kTile / 16; ++k) {
#pragma unroll
            for (int mb = 0; mb < 2; ++mb)
              tc::mma_bf16(tmem + o_col + mb * kN, dV + ((((mb ? s3 : s2) * C::kHalfBytes) + k * 16 * 128) >> 4),
                           b0 + (((k >> 2) * kN * 128 + (k & 3) * 32) >> 4), idO, (!first || k > 0) ? 1u : 0u);
          }
          tc::mma_commit(&bars[kODone0 + (i & 1)]);
          tc::mma_commit(&bars[kKVEmpty0 + s2]);
          tc::mma_commit(&bars[kKVEmpty0 + s3]);
          if (last_o) tc::mma_commit(&bars[kOSeg0 + (o_seg & 1)]);
          if (i + 1 < n_local) wo.next(p);
          continue;
        }
        tc::fence_after_sync();
        const int st = i % C::kStages;
        const uint64_t a0 = dV + ((st * C::kKVBytes) >> 4);
        // O^T += V^T P^T: A = V^T (MN-major: head dim contiguous; 64-wide
        // blocks kTile*128 bytes apart), B = P^T (K-major over tokens).
#pragma unroll
        for (int k = 0; k < kTile / 16; ++k) {
#pragma unroll
          for (int mb = 0; mb < D / C::kMO; ++mb)
            tc::mma_bf16(tmem + o_col + mb * kN, a0 + ((mb * (C::kMO / 64) * kTile * 128 + k * 16 * 128) >> 4),
                         b0 + (((k >> 2) * kN * 128 + (k & 3) * 32) >> 4), idO, (!first || k > 0) ? 1u : 0u);
        }
        tc::mma_commit(&bars[kODone0 + (i & 1)]);
        tc::mma_commit(&bars[kKVEmpty0 + st]);
        if (last_o) tc::mma_commit(&bars[kOSeg0 + (o_seg & 1)]);
        if (i + 1 < n_local) wo.next(p);
      }
    }
  } else if (warp < 4) {
    // ------------------------------------------------------------ softmax
    const int t = tid;  // token row of the tile == TMEM lane
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    Walker w;
    w.start(p, s0, pre0, t0, len0, pbeg0);
    float m_ref[NREP], l_tok[NREP];
    int seg = -1;
    bool ok = true;
    for (int i = 0; i < n_local; ++i) {
      const bool first = (i == 0) || w.j == 0;
      const bool last = (i == n_local - 1) || w.j == w.T - 1;
      if (first) {
        ++seg;
#pragma unroll
        for (int h = 0; h < NREP; ++h) {
          m_ref[h] = -INFINITY;
          l_tok[h] = 0.0f;
        }
      }
      const uint32_t o_col = C::kTmemO + (seg & 1) * 32;
      ok = tc::wait_bounded(&bars[kSFull0 + (i & 1)], (i >> 1) & 1, abort_flag, p.err, 30);
      if (!ok) break;
      tc::fence_after_sync();
      float sv[16];
      tmem_ld16(lane_addr + C::kTmemS + (i & 1) * kN, sv);
      if (PREC && p.q_f32) {
#pragma unroll
        for (int h = 0; h < NREP; ++h) sv[h] += sv[h + 8];  // K.Q_hi + K.Q_lo
      }
      const bool valid = w.j * kTile + t < w.len;
      bool need = false;
#pragma unroll
      for (int h = 0; h < NREP; ++h) {
        sv[h] = valid ? sv[h] * p.qscale : -INFINITY;
        need |= (m_ref[h] == -INFINITY) || (sv[h] > m_ref[h] + kRescaleLog2);
      }
      // CTA-uniform: must a reference max move on this tile?  Usually not,
      // and then P = exp2(s - m_ref) <= 2^8 needs no exchange of maxima.
      const bool moved = tc::named_sync_or(1, 128, need);
      float alpha[NREP];
      bool rescale = false;
#pragma unroll
      for (int h = 0; h < NREP; ++h) alpha[h] = 1.0f;
      if (moved) {
        float* rm = red_max + (i & 1) * 4 * kN;
#pragma unroll
        for (int h = 0; h < NREP; ++h) {
          const float wm = warp_max(sv[h]);
          if (lane == 0) rm[warp * kN + h] = wm;
        }
        tc::named_sync(1, 128);
#pragma unroll
        for (int h = 0; h < NREP; ++h) {
          const float mt = fmaxf(fmaxf(rm[h], rm[kN + h]), fmaxf(rm[2 * kN + h], rm[3 * kN + h]));
          if (mt > m_ref[h] + kRescaleLog2 || m_ref[h] == -INFINITY) {  // CTA-uniform decision
            alpha[h] = (m_ref[h] == -INFINITY) ? 0.0f : exp2f(m_ref[h] - mt);
            m_ref[h] = mt;  // finite: every tile holds a valid token
            rescale |= !first;
          }
        }
      }
#pragma unroll
      for (int h = 0; h < NREP; ++h) {
        sv[h] = exp2f(sv[h] - m_ref[h]);  // masked tokens: exp2(-inf) = 0
        l_tok[h] = l_tok[h] * alpha[h] + sv[h];
      }
      if (rescale) {
        // O^T is current once the previous P V finishes (and with it every
        // earlier one, so P^T buffer i&1 is free too).
        ok = tc::wait_bounded(&bars[kODone0 + ((i - 1) & 1)], ((i - 1) >> 1) & 1, abort_flag, p.err, 31);
        if (!ok) break;
        tc::fence_after_sync();
        {
#pragma unroll
          for (int mb = 0; mb < D / C::kMO; ++mb) {
            float ov[16];
            tmem_ld16(lane_addr + o_col + mb * kN, ov);
#pragma unroll
            for (int h = 0; h < NREP; ++h) {
              ov[h] *= alpha[h];
              if constexpr (PREC) ov[h + 8] *= alpha[h];
            }
            tmem_st16(lane_addr + o_col + mb * kN, ov);
          }
          tc::tmem_st_wait();
        }
      } else if (i >= 2) {
        // P^T buffer i&1 is free once the P V of tile i-2 finishes.
        ok = tc::wait_bounded(&bars[kODone0 + (i & 1)], ((i - 2) >> 1) & 1, abort_flag, p.err, 33);
        if (!ok) break;
      }
      // P^T[h][t] (bf16) in the K-major swizzled layout: 64-token sub-tiles
      // of 16 rows x 128 bytes; 16-byte chunk index XOR (row % 8).
      {
        const int sub = t >> 6, col = t & 63;
#pragma unroll
        for (int h = 0; h < NREP; ++h) {
          const int off = sub * (kN * 128) + h * 128 + ((((col >> 3) ^ (h & 7))) << 4) + (col & 7) * 2;
          const __nv_bfloat16 hi = __float2bfloat16_rn(sv[h]);
          *reinterpret_cast<__nv_bfloat16*>(p_s + (i & 1) * C::kPBytes + off) = hi;
          if constexpr (PREC)  // row h + 8: the remainder (same swizzle phase)
            *reinterpret_cast<__nv_bfloat16*>(p_s + (i & 1) * C::kPBytes + off + 8 * 128) =
                __float2bfloat16_rn(sv[h] - __bfloat162float(hi));
        }
      }
      // One arrival per softmax warp instead of 128 on one mbarrier word:
      // each lane fences its P^T stores to the async proxy, the warp
      // converges, lane 0 arrives.
      fence_proxy_async_shared();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&bars[kPFull0 + (i & 1)]);

      if (last) {
        // ---- hand the segment to the epilogue warps: per-warp row sums and
        // the reference maxima into slot seg & 1.  The slot (and O^T buffer
        // seg & 1) is free once the epilogue of segment seg - 2 has read it.
        if (seg >= 2) {
          bool fr = true;
          if (lane == 0) fr = tc::wait_bounded(&bars[kOFree0 + (seg & 1)], ((seg >> 1) - 1) & 1, abort_flag, p.err, 34);
          ok = __shfl_sync(0xffffffffu, fr, 0);
          if (!ok) break;
        }
        float* rl = red_l + (seg & 1) * 4 * kN;
#pragma unroll
        for (int h = 0; h < NREP; ++h) {
          const float wsum = warp_sum(l_tok[h]);
          if (lane == 0) rl[warp * kN + h] = wsum;
        }
        if (warp == 0 && lane == 0) {
#pragma unroll
          for (int h = 0; h < NREP; ++h) red_m[(seg & 1) * kN + h] = m_ref[h];
        }
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bars[kEFull0 + (seg & 1)]);
      }
      if (i + 1 < n_local) w.next(p);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Warps 6-9: warp w reads TMEM lanes 32 (w % 4) .. +31, so the four
    // cover O^T's 128 lanes.  Segment k's epilogue waits for its softmax
    // state (kEFull) and its last P V (kOSeg), reads O^T, then frees the
    // buffer (kOFree) before the global stores.
    const int t = tid - kEpiWarp0 * 32;  // 0 .. 127
    const int quarter = warp & 3;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    // Rows of O^T this thread holds: M=64 puts row d in lane (d % 16) + 32 (d / 16);
    // M=128 puts row d in lane d; D = 256 uses two M=128 blocks 16 columns apart.
    const bool holds = (C::kMO == 64) ? (lane < 16) : true;
    const int d_base = (C::kMO == 64) ? quarter * 16 + lane : quarter * 32 + lane;
    grid_wait();
    empty_outputs();
    Walker w;
    w.start(p, s0, pre0, t0, len0, pbeg0);
    int seg = -1;
    int n_pend = 0;  // partial segments written (at most the first and the last)
    bool early = false;             // pend[0] already holds its ticket (thread 0)
    unsigned int early_ticket = 0;  // that ticket
    bool ok = true;
    for (int i = 0; i < n_local; ++i) {
      const bool first = (i == 0) || w.j == 0;
      const bool last = (i == n_local - 1) || w.j == w.T - 1;
      if (first) ++seg;
      if (last) {
        const int b = seg & 1;
        bool good = tc::wait_bounded(&bars[kEFull0 + b], (seg >> 1) & 1, abort_flag, p.err, 40) &&
                    tc::wait_bounded(&bars[kOSeg0 + b], (seg >> 1) & 1, abort_flag, p.err, 41);
        good = __all_sync(0xffffffffu, good);  // warp-uniform for tcgen05.ld
        ok = !tc::named_sync_or(3, 128, !good);  // and uniform over the four warps
        if (!ok) break;
        tc::fence_after_sync();
        const uint32_t o_col = C::kTmemO + b * 32;
        float ov[D / C::kMO][16];
#pragma unroll
        for (int mb = 0; mb < D / C::kMO; ++mb) {
          tmem_ld16(lane_addr + o_col + mb * kN, ov[mb]);
          if constexpr (PREC) {
#pragma unroll
            for (int h = 0; h < NREP; ++h) ov[mb][h] += ov[mb][h + 8];  // V.P_hi + V.P_lo
          }
        }
        float l_cta[NREP], m_seg[NREP];
        const float* rl = red_l + b * 4 * kN;
#pragma unroll
        for (int h = 0; h < NREP; ++h) {
          l_cta[h] = rl[h] + rl[kN + h] + rl[2 * kN + h] + rl[3 * kN + h];
          m_seg[h] = red_m[b * kN + h];
        }
        tc::fence_before_sync();
        tc::mbar_arrive(&bars[kOFree0 + b]);  // O^T buffer and sums slot reusable two segments on
        const int64_t head0 = static_cast<int64_t>(w.s) * p.hq + w.g * NREP;
        const int64_t s_start = w.seg_start(p);
        const int64_t ca = cta_of(bnd, s_start, U, ctas), cb = cta_of(bnd, s_start + w.T - 1, U, ctas);
        if (ca == cb) {
          if (holds) {
#pragma unroll
            for (int mb = 0; mb < D / C::kMO; ++mb)
#pragma unroll
              for (int h = 0; h < NREP; ++h)
                store_out(p, (head0 + h) * D + d_base + mb * 128,
                          finalize(ov[mb][h], l_cta[h], m_seg[h], p.phantom));
          }
          if constexpr (LSE) {
#pragma unroll
            for (int h = 0; h < NREP; ++h)
              if (t == h) p.lse[head0 + h] = row_lse(p.phantom, m_seg[h], l_cta[h]);  // one thread per head
          }
        } else {
          // Partial: slot (cta, 0) if the segment is this CTA's first, else (cta, 1).
          const int which = (cta == ca && t0 != s_start) ? 1 : 0;
          const int64_t slot = (cta * 2 + which) * kN;
          if (holds) {
#pragma unroll
            for (int mb = 0; mb < D / C::kMO; ++mb)
#pragma unroll
              for (int h = 0; h < NREP; ++h) p.ws_o[(slot + h) * D + d_base + mb * 128] = ov[mb][h];
          }
#pragma unroll
          for (int h = 0; h < NREP; ++h) {
            if (t == h) {  // static register indexing: one thread per head
              p.ws_ml[(slot + h) * 2 + 0] = m_seg[h];
              p.ws_ml[(slot + h) * 2 + 1] = l_cta[h];
            }
          }
          const int seg_id = static_cast<int>(static_cast<int64_t>(w.s) * p.hkv + w.g);
          if (t == 0) {
            const int wa = (tile_begin(bnd, ca, U, ctas) != s_start) ? 1 : 0;
            pend[n_pend] = make_int4(seg_id, static_cast<int>(ca), static_cast<int>(cb), wa);
          }
          if (cta == cb && i + 1 < n_local) {
            // The tail of a segment whose other pieces end their CTAs' ranges:
            // take the ticket now (those CTAs arrive later), so that at most
            // one merge is left for the end.  Only thread 0 waits on the fence;
            // the ticket value is first needed after the last tile.
            tc::named_sync(3, 128);  // every thread's partial is written
            if (t == 0) early_ticket = ticket_add(&p.ws_cnt[seg_id]);
            early = true;
          }
          ++n_pend;
        }
      }
      if (i + 1 < n_local) w.next(p);
    }

    // ---- deferred merges: one ticket per partial segment not yet ticketed
    // (both in one round trip); the last CTA to arrive merges the pieces in
    // CTA order.
    if (ok && n_pend > 0) {
      tc::named_sync(3, 128);  // pend[] and this CTA's partials are complete
      if (t < n_pend) {
        const int4 pd = pend[t];
        unsigned int ticket;
        if (t == 0 && early) {
          ticket = early_ticket;
        } else {
          ticket = ticket_add(&p.ws_cnt[pd.x]);
        }
        last_flag[t] = (ticket == static_cast<unsigned int>(pd.z - pd.y)) ? 1 : 0;
      }
      tc::named_sync(3, 128);
    }
    for (int pi = 0; ok && pi < n_pend; ++pi) {
      if (!last_flag[pi]) continue;
      const int4 pd = pend[pi];
      const int s = pd.x / p.hkv, g = pd.x - (pd.x / p.hkv) * p.hkv;
      const int64_t head0 = static_cast<int64_t>(s) * p.hq + g * NREP;
      const int ca = pd.y, np = pd.z - pd.y + 1, wa = pd.w;
      constexpr int kElems = (NREP * D + 127) / 128;
      // Pieces per round (one round trip each); 2 at 16 elements per thread,
      // so the merge stays within the registers of a 320-thread CTA.
      constexpr int kChunk = kElems > 8 ? 2 : 4;
      float* stage = reinterpret_cast<float*>(p_s);  // [kChunk][16][2] (m, l) in the idle P^T buffer
      float mrun[kElems], orun[kElems], lrun[kElems];
#pragma unroll
      for (int q = 0; q < kElems; ++q) {
        mrun[q] = -INFINITY;
        orun[q] = 0.0f;
        lrun[q] = 0.0f;
      }
      for (int kb = 0; kb < np; kb += kChunk) {
        const int nk = min(kChunk, np - kb);
        // This round's O loads and (m, l) loads all in flight together.
        float ov4[kElems][kChunk];
#pragma unroll
        for (int q = 0; q < kElems; ++q) {
          const int e = t + q * 128;
          const int h = e / D, d = e - (e / D) * D;
#pragma unroll
          for (int u = 0; u < kChunk; ++u) {
            const int k = kb + u;
            ov4[q][u] = 0.0f;
            if (e < NREP * D && u < nk) {
              const int64_t sl = (static_cast<int64_t>(ca + k) * 2 + (k == 0 ? wa : 0)) * kN + h;
              ov4[q][u] = ld_cg(p.ws_o + sl * D + d);
            }
          }
        }
        float2 ml = make_float2(-INFINITY, 0.0f);
        const int mk_ = t / NREP, mh = t - (t / NREP) * NREP;
        if (t < nk * NREP) {
          const int k = kb + mk_;
          const int64_t sl = (static_cast<int64_t>(ca + k) * 2 + (k == 0 ? wa : 0)) * kN + mh;
          ml = __ldcg(reinterpret_cast<const float2*>(p.ws_ml + sl * 2));
        }
        if (t < nk * NREP) {
          stage[(mk_ * kN + mh) * 2 + 0] = ml.x;
          stage[(mk_ * kN + mh) * 2 + 1] = ml.y;
        }
        tc::named_sync(3, 128);
#pragma unroll
        for (int q = 0; q < kElems; ++q) {
          const int e = t + q * 128;
          if (e >= NREP * D) continue;
          const int h = e / D;
          float mc = -INFINITY;
#pragma unroll
          for (int u = 0; u < kChunk; ++u)
            if (u < nk) mc = fmaxf(mc, stage[(u * kN + h) * 2]);
          if (mc == -INFINITY) continue;
          const float mnew = fmaxf(mrun[q], mc);
          const float a_old = (mrun[q] == -INFINITY) ? 0.0f : exp2f(mrun[q] - mnew);
          orun[q] *= a_old;
          lrun[q] *= a_old;
          mrun[q] = mnew;
#pragma unroll
          for (int u = 0; u < kChunk; ++u) {
            if (u >= nk) break;
            const float mk = stage[(u * kN + h) * 2];
            if (mk == -INFINITY) continue;
            const float a = exp2f(mk - mnew);
            orun[q] += ov4[q][u] * a;
            lrun[q] += stage[(u * kN + h) * 2 + 1] * a;
          }
        }
        tc::named_sync(3, 128);  // the stage is rewritten by the next round
      }
#pragma unroll
      for (int q = 0; q < kElems; ++q) {
        const int e = t + q * 128;
        if (e < NREP * D) {
          store_out(p, head0 * D + e, finalize(orun[q], lrun[q], mrun[q], p.phantom));
          if constexpr (LSE) {
            if (e % D == 0) p.lse[head0 + e / D] = row_lse(p.phantom, mrun[q], lrun[q]);
          }
        }
      }
      if (t == 0) p.ws_cnt[pd.x] = 0u;  // ready for the next call on this workspace
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, C::kTmemCols);
  }
}

template <int D, int NREP, bool PREC, bool LSE = false>
int launch_decode(const CUtensorMap& tkv, const CUtensorMap& tq, const DecodeParams& prm, cudaStream_t stream) {
  using C = DCfg<D>;
  auto kern = paged_decode_kernel<D, NREP, PREC, LSE>;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int grid = sm_count() * C::kCtasPerSm;
  const int smem = C::kSmem + (grid + 1) * 4;  // + the plan's CTA boundary table
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    MTN_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                 "cudaFuncSetAttribute(decode)");
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  // Programmatic dependent launch: this grid may begin while the previous
  // kernel of the stream finishes, if that kernel allows it (decode launches
  // do); the kernel waits for it before touching its data.
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  MTN_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, tkv, tq, prm), "cudaLaunchKernelEx(paged_decode_kernel)");
  return check_launch("paged_decode_kernel");
}

template <int D, bool PREC, bool LSE = false>
int dispatch_nrep(int nrep, const CUtensorMap& tkv, const CUtensorMap& tq, const DecodeParams& prm,
                  cudaStream_t stream) {
  switch (nrep) {
    case 1: return launch_decode<D, 1, PREC, LSE>(tkv, tq, prm, stream);
    case 2: return launch_decode<D, 2, PREC, LSE>(tkv, tq, prm, stream);
    case 3: return launch_decode<D, 3, PREC, LSE>(tkv, tq, prm, stream);
    case 4: return launch_decode<D, 4, PREC, LSE>(tkv, tq, prm, stream);
    case 5: return launch_decode<D, 5, PREC, LSE>(tkv, tq, prm, stream);
    case 6: return launch_decode<D, 6, PREC, LSE>(tkv, tq, prm, stream);
    case 7: return launch_decode<D, 7, PREC, LSE>(tkv, tq, prm, stream);
    case 8: return launch_decode<D, 8, PREC, LSE>(tkv, tq, prm, stream);
    default: return set_error(MTN_EINVAL, "paged decode: query heads per kv head %d not in [1,8]", nrep);
  }
}

template <int D>
int dispatch_prec(bool prec, int nrep, const CUtensorMap& tkv, const CUtensorMap& tq, const DecodeParams& prm,
                  cudaStream_t stream) {
  if (prm.lse != nullptr)  // shared-prefix decode: bf16 operands only (checked by the caller)
    return dispatch_nrep<D, false, true>(nrep, tkv, tq, prm, stream);
  return prec ? dispatch_nrep<D, true>(nrep, tkv, tq, prm, stream) : dispatch_nrep<D, false>(nrep, tkv, tq, prm, stream);
}

int decode_ctas(int head_dim) {
  const int per = head_dim == 64 ? DCfg<64>::kCtasPerSm : head_dim == 128 ? DCfg<128>::kCtasPerSm
                                                                          : DCfg<256>::kCtasPerSm;
  return sm_count() * per;
}

}  // namespace
}  // namespace mtn

using mtn::set_error;

namespace mtn {
namespace {

size_t plan_words(int grid) { return 4 + static_cast<size_t>(kPlanEntry) * grid + grid + 1; }

// Cost-balanced split of the tiles (laid end to end: sequence by sequence,
// kv head by kv head) into the CTAs' contiguous ranges.  A tile costs 8 and
// a segment start ((sequence, kv head) first tile) 16 more: a CTA whose range
// spans two segments pays a second epilogue, measured with %globaltimer at
// about two tiles of streaming.  The segment cost is used only with at least
// 25/8 tiles per CTA; then boundary targets are at least 25 cost units apart
// while tile starts are at most 24 apart, so boundaries strictly increase.
void split_tiles(const std::vector<int64_t>& T, int hkv, int64_t U, int64_t ctas, int32_t* bnd) {
  if (U <= ctas) {
    for (int64_t c = 0; c <= ctas; ++c) bnd[c] = static_cast<int32_t>(c);
    return;
  }
  const int64_t w8 = 8 * U >= 25 * ctas ? 16 : 0;
  int64_t ne = 0, tiles = 0;
  for (int64_t t : T) {
    ne += t > 0;
    tiles += t;
  }
  const int64_t ctot = (8 * tiles + w8 * ne) * hkv;
  size_t s = 0;
  int64_t acc = 0, pre = 0;
  for (int64_t c = 0; c < ctas; ++c) {
    const int64_t y = c * ctot / ctas;
    int64_t seg = 0;
    for (;;) {  // y < ctot: stops at a sequence with tiles
      seg = 8 * T[s] + (T[s] > 0 ? w8 : 0);
      if (y < acc + seg * hkv) break;
      acc += seg * hkv;
      pre += T[s];
      ++s;
    }
    const int64_t local = y - acc, g = local / seg, r = local - g * seg;
    // tile j of a segment starts at cost 0 (j = 0) or w8 + 8 j (j >= 1)
    const int64_t j = r == 0 ? 0 : std::max<int64_t>(1, (r - w8 + 7) / 8);
    bnd[c] = static_cast<int32_t>(pre * hkv + g * T[s] + std::min(j, T[s]));
  }
  bnd[ctas] = static_cast<int32_t>(U);
}

}  // namespace
}  // namespace mtn

extern "C" {

size_t mtn_paged_decode_plan_bytes(int32_t head_dim) {
  if (head_dim != 64 && head_dim != 128 && head_dim != 256) return 0;
  return (mtn::plan_words(mtn::decode_ctas(head_dim)) * 4 + 255) & ~static_cast<size_t>(255);
}

int mtn_paged_decode_plan(const int32_t* kv_indptr, const int32_t* seq_lens, int32_t n_seqs, int32_t page_size,
                          int32_t num_kv_heads, int32_t head_dim, void* plan, size_t plan_bytes) {
  MTN_CHECK_ARG(n_seqs >= 0 && page_size > 0 && num_kv_heads > 0, "mtn_paged_decode_plan: bad sizes");
  MTN_CHECK_ARG(n_seqs == 0 || (kv_indptr && seq_lens), "mtn_paged_decode_plan: null metadata");
  const size_t need = mtn_paged_decode_plan_bytes(head_dim);
  MTN_CHECK_ARG(need > 0, "mtn_paged_decode_plan: head_dim %d not in {64,128,256}", head_dim);
  MTN_CHECK_ARG(plan != nullptr && plan_bytes >= need, "mtn_paged_decode_plan: plan buffer of %zu bytes < %zu",
                plan_bytes, need);
  const int grid = mtn::decode_ctas(head_dim);
  // Valid lengths clamped to each block table, as the kernel clamps them.
  std::vector<int64_t> T(static_cast<size_t>(n_seqs)), len(static_cast<size_t>(n_seqs));
  int64_t tiles = 0;
  for (int32_t s = 0; s < n_seqs; ++s) {
    const int64_t cap = static_cast<int64_t>(kv_indptr[s + 1] - kv_indptr[s]) * page_size;
    len[s] = std::min<int64_t>(std::max<int64_t>(seq_lens[s], 0), std::max<int64_t>(cap, 0));
    T[s] = (len[s] + mtn::kTile - 1) / mtn::kTile;
    tiles += T[s];
  }
  const int64_t U = tiles * num_kv_heads;
  MTN_CHECK_ARG(U < (int64_t(1) << 31), "mtn_paged_decode_plan: %lld tiles exceed the plan's int32 range",
                static_cast<long long>(U));
  const int64_t ctas = std::min<int64_t>(grid, U);
  int32_t* w = static_cast<int32_t*>(plan);
  std::memset(w, 0, need);
  w[0] = mtn::kPlanMagic;
  w[1] = static_cast<int32_t>(ctas);
  w[2] = grid;
  w[3] = static_cast<int32_t>(U);
  int32_t* bnd = w + 4 + mtn::kPlanEntry * grid;
  if (ctas > 0) mtn::split_tiles(T, num_kv_heads, U, ctas, bnd);
  for (int64_t c = ctas + 1; c <= grid; ++c) bnd[c] = static_cast<int32_t>(U);
  int32_t s = 0;
  int64_t pre = 0;
  for (int64_t c = 0; c < ctas; ++c) {
    const int64_t t0 = bnd[c];
    while ((pre + T[s]) * num_kv_heads <= t0) {  // the sequence holding tile t0
      pre += T[s];
      ++s;
    }
    int32_t* e = w + 4 + mtn::kPlanEntry * c;
    e[0] = static_cast<int32_t>(t0);
    e[1] = bnd[c + 1] - bnd[c];
    e[2] = s;
    e[3] = static_cast<int32_t>(pre);
    e[4] = static_cast<int32_t>(len[s]);
    e[5] = kv_indptr[s];
  }
  return MTN_OK;
}

size_t mtn_paged_decode_workspace_bytes(int32_t n_seqs, int32_t num_q_heads, int32_t num_kv_heads,
                                        int32_t head_dim) {
  (void)num_q_heads;
  if (n_seqs <= 0 || num_kv_heads <= 0 || (head_dim != 64 && head_dim != 128 && head_dim != 256)) return 0;
  const int64_t slots = static_cast<int64_t>(mtn::decode_ctas(head_dim)) * 2 * mtn::kN;
  size_t bytes = static_cast<size_t>(slots) * head_dim * 4;    // ws_o
  bytes += static_cast<size_t>(slots) * 2 * 4;                   // ws_ml
  bytes += static_cast<size_t>(n_seqs) * num_kv_heads * 4;       // ws_cnt
  return (bytes + 255) & ~static_cast<size_t>(255);
}

int mtn_paged_decode_with_plan(const mtn_kv_layout* pool, int32_t layer, const void* q, int32_t q_dtype, void* o,
                               int32_t o_dtype, const void* k_new, const void* v_new, int32_t new_dtype,
                               int32_t n_seqs, int32_t num_q_heads, const int32_t* kv_indptr,
                               const int32_t* kv_indices, const int32_t* seq_lens, float scale, uint32_t flags,
                               const void* plan, void* workspace, size_t workspace_bytes, void* stream) {
  return mtn::paged_decode_impl(pool, layer, q, q_dtype, o, o_dtype, k_new, v_new, new_dtype, n_seqs, num_q_heads,
                                kv_indptr, kv_indices, seq_lens, scale, flags, plan, workspace, workspace_bytes,
                                stream, nullptr);
}

}  // extern "C"

int mtn::paged_decode_impl(const mtn_kv_layout* pool, int32_t layer, const void* q, int32_t q_dtype, void* o,
                           int32_t o_dtype, const void* k_new, const void* v_new, int32_t new_dtype, int32_t n_seqs,
                           int32_t num_q_heads, const int32_t* kv_indptr, const int32_t* kv_indices,
                           const int32_t* seq_lens, float scale, uint32_t flags, const void* plan, void* workspace,
                           size_t workspace_bytes, void* stream, float* lse) {
  int st = mtn::validate_layout(pool, layer, "mtn_paged_decode");
  if (st != MTN_OK) return st;
  MTN_CHECK_ARG(n_seqs >= 0, "mtn_paged_decode: n_seqs < 0");
  if (n_seqs == 0) return MTN_OK;
  MTN_CHECK_ARG(q && o && kv_indptr && kv_indices && seq_lens, "mtn_paged_decode: null pointer");
  MTN_CHECK_ARG(q_dtype == MTN_DTYPE_BF16 || q_dtype == MTN_DTYPE_F32, "mtn_paged_decode: bad q dtype");
  MTN_CHECK_ARG(o_dtype == MTN_DTYPE_BF16 || o_dtype == MTN_DTYPE_F32, "mtn_paged_decode: bad o dtype");
  MTN_CHECK_ARG((k_new == nullptr) == (v_new == nullptr), "mtn_paged_decode: give both k_new and v_new or neither");
  MTN_CHECK_ARG(k_new == nullptr || new_dtype == MTN_DTYPE_BF16 || new_dtype == MTN_DTYPE_F32,
                "mtn_paged_decode: bad k_new/v_new dtype");
  MTN_CHECK_ARG(num_q_heads > 0 && num_q_heads % pool->num_kv_heads == 0,
                "mtn_paged_decode: %d query heads not a multiple of %d kv heads", num_q_heads, pool->num_kv_heads);
  const int D = pool->head_dim;
  MTN_CHECK_ARG(pool->page_size % 8 == 0 && mtn::kTile % pool->page_size == 0,
                "mtn_paged_decode: page_size %d must be a multiple of 8 dividing %d", pool->page_size, mtn::kTile);
  MTN_CHECK_ARG((reinterpret_cast<uintptr_t>(q) & 15) == 0 && (reinterpret_cast<uintptr_t>(o) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(k_new) & 15) == 0 && (reinterpret_cast<uintptr_t>(v_new) & 15) == 0,
                "mtn_paged_decode: q/o/k_new/v_new must be 16-byte aligned");
  MTN_CHECK_ARG(static_cast<int64_t>(n_seqs) * num_q_heads < (int64_t(1) << 31), "mtn_paged_decode: q too large");
  const size_t need = mtn_paged_decode_workspace_bytes(n_seqs, num_q_heads, pool->num_kv_heads, D);
  MTN_CHECK_ARG(workspace != nullptr && workspace_bytes >= need,
                "mtn_paged_decode: workspace of %zu bytes < %zu needed", workspace_bytes, need);
  MTN_CHECK_ARG((reinterpret_cast<uintptr_t>(workspace) & 15) == 0, "mtn_paged_decode: workspace alignment");
  CUtensorMap tkv, tq;
  st = mtn::pool_tensor_map(pool, &tkv);
  if (st != MTN_OK) return st;
  if (q_dtype == MTN_DTYPE_BF16) {
    // 16-row boxes over the [n_seqs * heads, head_dim] view of q.
    st = mtn::q_tensor_map(q, static_cast<int64_t>(n_seqs) * num_q_heads, 1, D, mtn::kN, &tq);
    if (st != MTN_OK) return st;
  } else {
    std::memset(&tq, 0, sizeof(tq));
  }

  mtn::DecodeParams prm{};
  const int64_t rows_per_block = pool->num_pages * pool->num_kv_heads * pool->page_size;
  prm.row_k = (static_cast<int64_t>(layer) * 2 + 0) * rows_per_block;
  prm.row_v = (static_cast<int64_t>(layer) * 2 + 1) * rows_per_block;
  prm.pool = static_cast<__nv_bfloat16*>(pool->base);
  prm.num_pages = pool->num_pages;
  {
    // Boxes of pool_rows .. + page_size - 1 lie past the tensor (zero fill);
    // kept only while those coordinates fit TMA's signed 32-bit range.
    const int64_t rows = pool_rows(pool);
    prm.oob_row = rows + pool->page_size < (int64_t(1) << 31) ? static_cast<int>(rows) : -1;
  }
  prm.hkv = pool->num_kv_heads;
  prm.ps = pool->page_size;
  prm.hq = num_q_heads;
  prm.n_seqs = n_seqs;
  prm.q = q;
  prm.o = o;
  prm.q_f32 = q_dtype == MTN_DTYPE_F32;
  prm.o_f32 = o_dtype == MTN_DTYPE_F32;
  prm.k_new = k_new;
  prm.v_new = v_new;
  prm.new_f32 = new_dtype == MTN_DTYPE_F32;
  prm.kv_indptr = kv_indptr;
  prm.kv_indices = kv_indices;
  prm.seq_lens = seq_lens;
  prm.qscale = scale * mtn::kLog2e;
  prm.phantom = (flags & MTN_ATTN_PHANTOM_ZERO_SLOT) ? 1 : 0;
  const int64_t slots = static_cast<int64_t>(mtn::decode_ctas(D)) * 2 * mtn::kN;
  prm.ws_o = static_cast<float*>(workspace);
  prm.ws_ml = prm.ws_o + slots * D;
  prm.ws_cnt = reinterpret_cast<unsigned int*>(prm.ws_ml + slots * 2);
  prm.err = mtn::device_error_ptr();
  MTN_CHECK_ARG((reinterpret_cast<uintptr_t>(plan) & 15) == 0, "mtn_paged_decode: plan must be 16-byte aligned");
  prm.plan = static_cast<const int32_t*>(plan);
  prm.lse = lse;
  const int nrep = num_q_heads / pool->num_kv_heads;
  auto s = static_cast<cudaStream_t>(stream);
  const bool prec = (flags & MTN_ATTN_SPLIT_BF16) != 0;
  switch (D) {
    case 64: return mtn::dispatch_prec<64>(prec, nrep, tkv, tq, prm, s);
    case 128: return mtn::dispatch_prec<128>(prec, nrep, tkv, tq, prm, s);
    default: return mtn::dispatch_prec<256>(prec, nrep, tkv, tq, prm, s);
  }
}

extern "C" {

int mtn_paged_decode(const mtn_kv_layout* pool, int32_t layer, const void* q, int32_t q_dtype, void* o,
                     int32_t o_dtype, const void* k_new, const void* v_new, int32_t new_dtype, int32_t n_seqs,
                     int32_t num_q_heads, const int32_t* kv_indptr, const int32_t* kv_indices,
                     const int32_t* seq_lens, float scale, uint32_t flags, void* workspace, size_t workspace_bytes,
                     void* stream) {
  return mtn_paged_decode_with_plan(pool, layer, q, q_dtype, o, o_dtype, k_new, v_new, new_dtype, n_seqs, num_q_heads,
                                    kv_indptr, kv_indices, seq_lens, scale, flags, nullptr, workspace,
                                    workspace_bytes, stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free entry point: the workspace is mtn_noalloc_decode_scratch.

namespace {

constexpr size_t kNoAllocScratchBytes = sizeof(mtn_noalloc_decode_scratch);
std::mutex g_noalloc_mu;
void* g_noalloc_addr[64] = {};

// Device address of the scratch array on the current device, looked up once
// per device (with that device current).
int noalloc_scratch(void** out) {
  int dev = 0;
  MTN_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= 64) return mtn::set_error(MTN_EINVAL, "mtn_paged_decode_noalloc: device %d unsupported", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, mtn_noalloc_decode_scratch);
    if (e != cudaSuccess) return mtn::cuda_status(e, "cudaGetSymbolAddress(mtn_noalloc_decode_scratch)");
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return MTN_OK;
}

}  // namespace

extern "C" int mtn_paged_decode_noalloc(const mtn_kv_layout* pool, int32_t layer, const void* q, int32_t q_dtype,
                                        void* o, int32_t o_dtype, const void* k_new, const void* v_new,
                                        int32_t new_dtype, int32_t n_seqs, int32_t num_q_heads,
                                        const int32_t* kv_indptr, const int32_t* kv_indices,
                                        const int32_t* seq_lens, float scale, uint32_t flags, void* stream) {
  MTN_CHECK_ARG(pool != nullptr, "mtn_paged_decode_noalloc: null pool");
  MTN_CHECK_ARG(n_seqs >= 0, "mtn_paged_decode_noalloc: n_seqs < 0");
  if (n_seqs == 0) return MTN_OK;
  const int D = pool->head_dim;
  MTN_CHECK_ARG(D == 64 || D == 128 || D == 256, "mtn_paged_decode_noalloc: head_dim %d not in {64,128,256}", D);
  MTN_CHECK_ARG(pool->num_kv_heads > 0, "mtn_paged_decode_noalloc: bad pool");
  const size_t need = mtn_paged_decode_workspace_bytes(n_seqs, num_q_heads, pool->num_kv_heads, D);
  MTN_CHECK_ARG(need > 0 && need <= kNoAllocScratchBytes,
                "mtn_paged_decode_noalloc: %d sequences x %d kv heads need %zu bytes of scratch; the static scratch "
                "holds %zu (use mtn_paged_decode with a caller workspace)",
                n_seqs, pool->num_kv_heads, need, kNoAllocScratchBytes);
  void* scratch = nullptr;
  int st = noalloc_scratch(&scratch);
  if (st != MTN_OK) return st;
  // The arrival counters must start at zero.  Calls leave them zero, but a
  // call that failed part-way may not have: clear them on this stream.
  const int64_t slots = static_cast<int64_t>(mtn::decode_ctas(D)) * 2 * mtn::kN;
  const size_t cnt_off = static_cast<size_t>(slots) * (D + 2) * 4;
  const size_t cnt_bytes = static_cast<size_t>(n_seqs) * pool->num_kv_heads * 4;
  MTN_CUDA_TRY(cudaMemsetAsync(static_cast<unsigned char*>(scratch) + cnt_off, 0, cnt_bytes,
                               static_cast<cudaStream_t>(stream)),
               "cudaMemsetAsync(decode scratch counters)");
  return mtn_paged_decode(pool, layer, q, q_dtype, o, o_dtype, k_new, v_new, new_dtype, n_seqs, num_q_heads,
                          kv_indptr, kv_indices, seq_lens, scale, flags, scratch, kNoAllocScratchBytes, stream);
}
