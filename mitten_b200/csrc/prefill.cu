// Chunked-prefill attention over paged KV on the sm_100a tensor cores.
//
// Replaces the prefill-chunk attention of qwen model.rs:394-416 for a chunk
// of q_len new tokens appended after P cached ones: scores q.k * scale
// (model.rs:298, 413), causal mask -1e10 for keys after the query
// (generate_causal_mask, model.rs:542-555), softmax over every key plus the
// optional all-zero first row (model.rs:207-220), output P.V (model.rs:416),
// q head h reading kv head h / n_rep (model.rs:398-408).
//
// CTA = (128-row query tile, query head, sequence); 6 warps in 3 roles:
//   warps 0-3  softmax: one TMEM lane (= one query row) per thread.  They
//              first write the Q tile into TMEM as bf16 pairs (both
//              contractions take their M x K operand from TMEM, so the tensor
//              core reads only K and V from shared memory), then per KV tile:
//              online softmax in the exp2 domain against a per-row reference
//              max that moves only when a tile exceeds it by 2^8 (so the TMEM
//              O accumulator is rarely rescaled), and P written as bf16 pairs
//              over the first half of the tile's S columns; finally O / l.
//   warp 4     TMA producer: K and V pages of each KV tile (one 4-D box per
//              page covers every head-dim block) into a 3-stage ring with
//              separate K and V barriers; page ids fetched by the whole warp
//              one 32-page window ahead, straight from the block table.
//   warp 5     MMA issuer (one thread): S = Q K^T and O += P V with
//              tcgen05.mma (M=128, kind::f16, f32 accumulators in TMEM),
//              completion signalled with tcgen05.commit on mbarriers.  S is
//              double-buffered in TMEM: the next tile's Q K^T runs on the
//              tensor cores while the softmax works on this one.
// Every wait is bounded (~1 s); a timeout records kDevErrTimeout, releases
// the other roles, frees TMEM and returns.
#include <mutex>

#include "common.cuh"
#include "tc.cuh"
#include "tmaps.hpp"

namespace mtn {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kBM = 128;   // query rows per CTA (TMEM lanes)
constexpr int kThreads = 192;

struct PrefillParams {
  const void* q;  // [total_q][hq][head_dim], bf16 or (q_f32) f32
  int q_f32;
  const int32_t* qo_indptr;
  const int32_t* kv_indptr;
  const int32_t* kv_indices;
  const int32_t* seq_lens;
  void* o;
  int o_f32;
  int hq;
  int hkv;
  int ps;
  int64_t num_pages;
  int64_t row_k;  // row (of the pool's [rows, head_dim] view) of layer K, page 0, head 0, token 0
  int64_t row_v;
  float qscale;
  int phantom;
  int* err;
  // Used only by the shared-prefix decode (one-tile kernel): noncausal = every
  // query row sees every key of its sequence (the queries are other
  // sequences' tokens, all after the shared keys); lse = per (row, head)
  // log2-domain log-sum-exp of the row's softmax, [total_q][hq], or null.
  int noncausal;
  float* lse;
  // Non-causal launches have one pseudo-sequence given by scalars: nc_q_len
  // query rows over the nc_pages pages kv_indices[0 ..] (all tokens valid).
  int nc_q_len;
  int nc_pages;
  // Split of long units, for launches with few units: a (query tile, head,
  // sequence) unit is cut into k <= kMaxPieces pieces of consecutive kv
  // tiles, run by CTAs blockIdx.z = piece * n_seqs + sequence (pieces in the
  // slowest grid dimension, so every unit's first piece is dispatched before
  // any other).  Each piece leaves (O, m, l) in its workspace slot; the last
  // to arrive merges them.
  int split;
  int split_target;       // CTAs one wave holds (the SM count)
  int n_seqs;
  int64_t max_units;      // workspace units (unit index bound)
  float* ws_o;            // [units * kMaxPieces][D / 32][8][128 rows][4]
  float* ws_ml;           // [units * kMaxPieces][2][128 rows]: m, l
  unsigned int* ws_cnt;   // [units] arrival counters, left at zero
};

constexpr int kMaxPieces = 4;
constexpr int kMinPiece = 8;        // kv tiles
constexpr int kSplitMaxUnits = 296; // launches with more units run unsplit

// P is exponentiated against a per-row reference max that moves only when a
// tile's max exceeds it by more than 2^8, so P <= 256 and O is rarely rescaled.
constexpr float kRescaleLog2 = 8.0f;

template <int D>
struct PCfg {
  static constexpr int kBN = D <= 128 ? 128 : 64;       // kv tokens per tile
  static constexpr int kDB = D / 64;                    // 64-wide head-dim blocks
  static constexpr int kStages = 3;                     // K/V ring depth
  static constexpr int kKVBytes = kBN * D * 2;          // one of K or V per stage
  static constexpr int kGroupBytes = kDB * 1024;        // 8 kv rows, all head-dim blocks
  static constexpr int kOffK = 0;                       // [kStages][kKVBytes]
  static constexpr int kOffV = kOffK + kStages * kKVBytes;
  static constexpr int kOffBar = kOffV + kStages * kKVBytes;
  static constexpr int kOffMisc = kOffBar + 24 * 8;     // tmem base, abort flag
  static constexpr int kSmem = kOffMisc + 64 + 1024;    // + slack for 1024-byte alignment
  // TMEM columns: S[2] (P of a tile overwrites the first kBN/2 columns of its
  // S buffer as bf16 pairs; with split operands the remainder of P takes the
  // other kBN/2), the O accumulator, Q as bf16 pairs and, with split
  // operands, the remainder of Q after it (head_dim <= 128 only).
  static constexpr int kTmemS = 0;
  static constexpr int kTmemO = 2 * kBN;
  static constexpr int kTmemQ = 2 * kBN + D;
  static constexpr int kTmemQlo = kTmemQ + D / 2;
  static constexpr int kTmemCols = 512;
  static constexpr bool kSplitFits = kTmemQlo + D / 2 <= kTmemCols;
  static_assert(kTmemQ + D / 2 <= kTmemCols, "TMEM budget");
  static_assert(kSmem <= 227 * 1024, "shared memory");
};

enum Bar {
  kQReady = 0,    // Q in TMEM (128 softmax threads)
  kKFull0 = 1,    // [3] K of tile j landed in stage j%3
  kVFull0 = 4,    // [3]
  kKEmpty0 = 7,   // [3] S of tile j done: K stage free
  kVEmpty0 = 10,  // [3] P V of tile j done: V stage free
  kSFull0 = 13,   // [2] S buffer j&1 holds tile j's scores
  kPFull0 = 15,   // [2] P(j) written over S buffer j&1 (128 softmax threads)
  kODone0 = 17,   // [2] P V of tile j done: O current
  kNumBars = 19
};

// Piece length of the split, the same value in every CTA of the launch: the
// launch's units (query tile, head) and their kv tiles T, each unit's tiles
// being (last visible position / kBN) + 1; with U units on S SMs a piece
// length of T / (S - U) keeps every piece in one wave (sum of
// ceil(n / plen) < T / plen + U <= S).  0 when the units fill the SMs.
__device__ __forceinline__ int64_t split_piece_len(const PrefillParams& p, int bn, int lane) {
  int64_t t = 0, u = 0;
  if (p.noncausal) {
    if (lane == 0) {
      u = (p.nc_q_len + kBM - 1) / kBM;
      t = u * ((static_cast<int64_t>(p.nc_pages) * p.ps + bn - 1) / bn);
    }
  }
  for (int s = lane; !p.noncausal && s < p.n_seqs; s += 32) {
    const int q0 = p.qo_indptr[s];
    const int ql = p.qo_indptr[s + 1] - q0;
    if (ql <= 0) continue;
    const int64_t kl = max(static_cast<int64_t>(p.seq_lens[s]), static_cast<int64_t>(p.noncausal ? 1 : ql));
    for (int qt = 0; qt * kBM < ql; ++qt) {
      t += p.noncausal ? (kl + bn - 1) / bn : (kl - ql + min(ql, (qt + 1) * kBM) - 1) / bn + 1;
      ++u;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    t += __shfl_xor_sync(0xffffffffu, t, o);
    u += __shfl_xor_sync(0xffffffffu, u, o);
  }
  t *= p.hq;
  u *= p.hq;
  if (u >= p.split_target) return 0;
  // Non-causal launches (the shared-prefix part: few units, short) cut down
  // to 2-tile pieces; causal ones keep kMinPiece.
  const int64_t min_piece = p.noncausal ? 2 : kMinPiece;
  return max(min_piece, (t + (p.split_target - u) - 1) / (p.split_target - u));
}

// 1 / l for a row whose softmax has max m (log2 units) and sum l, with the
// phantom zero key (score 0, value 0) folded in when `phantom` is set; the
// returned factor also rescales O from m to the phantom-aware max.
__device__ __forceinline__ float row_inv_sum(int phantom, float m, float l) {
  float a = 1.0f;
  if (phantom) {
    const float mf = fmaxf(m, 0.0f);
    a = m == -INFINITY ? 0.0f : exp2f(m - mf);
    l = l * a + exp2f(-mf);
  }
  return l > 0.0f ? a / l : 0.0f;
}

// Store 32 consecutive head-dim values of one output row, scaled by inv.
__device__ __forceinline__ void store_row_chunk(const PrefillParams& p, int64_t elem0, const float* v, float inv) {
  if (p.o_f32) {
    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.o) + elem0);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      dst[i] = make_float4(v[4 * i] * inv, v[4 * i + 1] * inv, v[4 * i + 2] * inv, v[4 * i + 3] * inv);
  } else {
    uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.o) + elem0);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 w;
      w.x = f2_to_bf2(v[8 * i + 0] * inv, v[8 * i + 1] * inv);
      w.y = f2_to_bf2(v[8 * i + 2] * inv, v[8 * i + 3] * inv);
      w.z = f2_to_bf2(v[8 * i + 4] * inv, v[8 * i + 5] * inv);
      w.w = f2_to_bf2(v[8 * i + 6] * inv, v[8 * i + 7] * inv);
      dst[i] = w;
    }
  }
}

// One kv tile of the online softmax over a 128-row query tile, one row per
// thread (warp w of the four reads TMEM lanes 32 (w % 4) ..): wait for S on
// `sfull`, mask keys after the row's position on the diagonal tile, move the
// row's reference max only when the tile exceeds it by 2^8 (then rescale O
// in TMEM once the previous P V is done: `odone_prev`), write P as bf16
// pairs over the first kBN / 2 columns of the S buffer and arrive on
// `pfull`.  Returns false (every lane of the warp) when a wait gave up.
template <int D, int kBN, bool PREC = false>
__device__ __forceinline__ bool softmax_tile(uint32_t lane_base, uint32_t s_off, uint32_t o_off, int key0, int pos0,
                                             int row_pos, float qscale, float& m_ref, float& l_run, uint64_t* sfull,
                                             uint32_t s_par, uint64_t* odone_prev, uint32_t o_par, uint64_t* pfull,
                                             volatile int* abort_flag, int* err, int where) {
  bool ok = tc::wait_bounded(sfull, s_par, abort_flag, err, where);
  if (!__all_sync(0xffffffffu, ok)) return false;  // TMEM loads below are warp-collective
  tc::fence_after_sync();
  const uint32_t s_col = lane_base + s_off;
  float sv[kBN];
  {
    uint32_t r[kBN / 32][32];
#pragma unroll
    for (int c = 0; c < kBN / 32; ++c) tc::tmem_ld32(s_col + c * 32, r[c]);
    tc::tmem_ld_wait();
#pragma unroll
    for (int c = 0; c < kBN; ++c) sv[c] = __uint_as_float(r[c >> 5][c & 31]);
  }
  if (key0 + kBN - 1 > pos0) {  // diagonal tile: keys after a row's position are masked
#pragma unroll
    for (int c = 0; c < kBN; ++c) sv[c] = (key0 + c <= row_pos) ? sv[c] : -INFINITY;
  }
  // Row max of the raw scores in 8 independent chains, two scores per
  // three-input max (scale > 0 commutes with max).
  float mx[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) mx[i] = sv[i];
#pragma unroll
  for (int c = 8; c < kBN; c += 2) mx[(c >> 1) & 7] = tc::max3(mx[(c >> 1) & 7], sv[c], sv[c + 1]);
  const float mt =
      fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * qscale;
  // Lazy rescale, per row: the reference max moves only when this tile
  // exceeds it by 2^8.  A row's first tile always sets it when the row sees
  // a key there; a row that sees no key yet keeps m_ref = -inf with P = 0.
  float alpha = 1.0f;
  bool moved = false;
  if (m_ref == -INFINITY) {
    m_ref = mt;
  } else if (mt > m_ref + kRescaleLog2) {
    alpha = exp2f(m_ref - mt);
    m_ref = mt;
    moved = true;
  }
  const float neg_m = m_ref == -INFINITY ? 0.0f : -m_ref;
  float ps8[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) ps8[i] = 0.0f;
  // Pairs of scores through the packed f32x2 FMA and add: the same roundings
  // as one fmaf / add per score, and score c still sums into chain c & 7.
#pragma unroll
  for (int c = 0; c < kBN; c += 2) {
    float x0, x1;
    tc::fma2(x0, x1, sv[c], sv[c + 1], qscale, neg_m);
    sv[c] = tc::ex2_approx(x0);  // masked keys: 2^-inf = 0
    sv[c + 1] = tc::ex2_approx(x1);
    tc::add2(ps8[c & 7], ps8[(c & 7) + 1], sv[c], sv[c + 1]);
  }
  const float psum = ((ps8[0] + ps8[1]) + (ps8[2] + ps8[3])) + ((ps8[4] + ps8[5]) + (ps8[6] + ps8[7]));
  l_run = l_run * alpha + psum;
  // P (bf16 pairs) over the first kBN/2 columns of this tile's S buffer;
  // with split operands its remainders over the other kBN/2.
#pragma unroll
  for (int c = 0; c < kBN / 64; ++c) {
    uint32_t r[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) r[i] = f2_to_bf2(sv[c * 64 + 2 * i], sv[c * 64 + 2 * i + 1]);
    tc::tmem_st32(s_col + c * 32, r);
    if constexpr (PREC) {
#pragma unroll
      for (int i = 0; i < 32; ++i) r[i] = bf2_residual(r[i], sv[c * 64 + 2 * i], sv[c * 64 + 2 * i + 1]);
      tc::tmem_st32(s_col + kBN / 2 + c * 32, r);
    }
  }
  tc::tmem_st_wait();
  if (__any_sync(0xffffffffu, moved)) {
    // O is current once P V of the previous tile finishes (P is stored
    // first, so the 128 exponentials are no longer live here).
    ok = tc::wait_bounded(odone_prev, o_par, abort_flag, err, where + 1);
    if (!__all_sync(0xffffffffu, ok)) return false;
    tc::fence_after_sync();
#pragma unroll 1
    for (int c = 0; c < D / 32; ++c) {
      uint32_t r[32];
      tc::tmem_ld32(lane_base + o_off + c * 32, r);
      tc::tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
      tc::tmem_st32(lane_base + o_off + c * 32, r);
    }
    tc::tmem_st_wait();
  }
  tc::fence_before_sync();
  tc::mbar_arrive(pfull);
  return true;
}

// PREC (MTN_ATTN_SPLIT_BF16): Q and P as bf16 hi + lo pairs, hi = bf16(x)
// and lo = bf16(x - hi); S = Q_hi K^T + Q_lo K^T and O += P_hi V + P_lo V,
// all accumulated in the same f32 TMEM columns (twice the MMAs).
template <int D, bool PREC>
__global__ void __launch_bounds__(kThreads, 1)
    paged_prefill_kernel(const __grid_constant__ CUtensorMap tm_kv, const __grid_constant__ PrefillParams p) {
  using C = PCfg<D>;
  static_assert(!PREC || C::kSplitFits, "split operands need head_dim <= 128");
  constexpr int kS = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tile = blockIdx.x, h = blockIdx.y;
  const int piece = p.split ? static_cast<int>(blockIdx.z) / p.n_seqs : 0;
  const int s = static_cast<int>(blockIdx.z) - piece * p.n_seqs;
  // With the split on, the MMA warp (idle until the pipeline starts) computes
  // the launch's piece length while the other warps load this unit's
  // metadata, so the two global round trips overlap.
  int64_t* plen_s = reinterpret_cast<int64_t*>(smem + C::kOffMisc + 16);
  const bool scan_warp = p.split && warp == 5;
  if (scan_warp) {
    const int64_t pl = split_piece_len(p, C::kBN, lane);
    if (lane == 0) *plen_s = pl;
  }
  int q0 = 0, q_len = 0, kv_beg = 0, npages = 0, kv_len = 0;
  auto load_meta = [&]() {
    if (p.noncausal) {
      q0 = 0;
      q_len = p.nc_q_len;
      kv_beg = 0;
      npages = p.nc_pages;
      kv_len = p.nc_pages * p.ps;
      return;
    }
    q0 = p.qo_indptr[s];
    q_len = p.qo_indptr[s + 1] - q0;
    kv_beg = p.kv_indptr[s];
    npages = p.kv_indptr[s + 1] - kv_beg;
    kv_len = p.seq_lens[s];
  };
  if (!scan_warp) load_meta();
  if (p.split) __syncthreads();
  if (scan_warp) load_meta();
  if (tile * kBM >= q_len) return;
  const int min_kv = p.noncausal ? 1 : q_len;  // non-causal rows need at least one key
  if (kv_len < min_kv || kv_len > npages * p.ps) {
    if (tile == 0 && h == 0 && piece == 0 && threadIdx.x == 0) record_error(p.err, kDevErrBadSeqLen, s);
    kv_len = max(min_kv, min(kv_len, npages * p.ps));
    if (kv_len > npages * p.ps) return;  // not even the chunk fits its pages
  }
  const int nrows = min(kBM, q_len - tile * kBM);
  // Position of row 0 and of the last row; non-causal rows all sit after
  // the last key, so only keys past kv_len are masked.
  const int pos0 = p.noncausal ? kv_len - 1 : kv_len - q_len + tile * kBM;
  const int last_pos = p.noncausal ? kv_len - 1 : pos0 + nrows - 1;
  const int n_tiles = last_pos / C::kBN + 1;
  const int g = h / (p.hq / p.hkv);
  const int pages_per_tile = C::kBN / p.ps;
  // Unit index for the split's workspace: q0 / 128 + s + tile is distinct
  // per (sequence, query tile) and below total_q / 128 + n_seqs.
  const int64_t uid = (static_cast<int64_t>(q0 / kBM) + s + tile) * p.hq + h;
  int k = 1;  // pieces of this unit
  if (p.split && uid < p.max_units) {
    const int64_t plen = *plen_s;
    if (plen > 0) k = static_cast<int>(min(static_cast<int64_t>(kMaxPieces), (n_tiles + plen - 1) / plen));
  }
  if (piece >= k) return;
  const int ja = piece * n_tiles / k;  // this CTA's kv tiles [ja, jb)
  const int jb = (piece + 1) * n_tiles / k;
  const int nt = jb - ja;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i)
      mbar_init(&bars[i], (i == kQReady || i == kPFull0 || i == kPFull0 + 1) ? kBM : 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(tmem_base_s, C::kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_base_s;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    // One 4-D box per page brings a page of this kv head, all head-dim
    // blocks, as [8-row groups][64-column blocks][8 rows][128 bytes]; the
    // pages of a tile sit back to back, so every 8-row group of the tile is
    // kGroupBytes after the previous one.  K of a stage is refilled once S of
    // the tile kStages back is done, V once its P V is done.  Page ids are
    // fetched by the whole warp, 32 at a time and one window ahead, so no
    // load of the block table sits on the issue path; lane 0 issues.
    const int ppt = pages_per_tile;
    const int pb = ja * ppt;                    // first page of the range
    const int lim = min(npages, jb * ppt) - 1;  // last page the CTA reads
    auto fetch = [&](int first) -> int { return p.kv_indices[kv_beg + min(first + lane, lim)]; };
    auto to_row = [&](int page) -> int {  // first pool row / 8 of this kv head's slice of the page (K)
      if (page < 0 || page >= p.num_pages) {
        record_error(p.err, kDevErrBadPage, s);
        page = 0;
      }
      return static_cast<int>((p.row_k + (static_cast<int64_t>(page) * p.hkv + g) * p.ps) >> 3);
    };
    if (lane == 0) tc::prefetch_tmap(&tm_kv);
    const int page_bytes = p.ps * D * 2;
    const int dv = static_cast<int>((p.row_v - p.row_k) >> 3);
    int cur = to_row(fetch(pb));
    int nxt = fetch(pb + 32);
    for (int j = 0; j < nt; ++j) {  // j counts the range's tiles
      const int st = j % kS;
      const uint32_t par = ((j / kS) - 1) & 1;  // phase of the use kStages tiles back
      const int first = j * ppt;                 // page offset inside the range
      if (j > 0 && (first & 31) == 0) {
        cur = to_row(nxt);
        nxt = fetch(pb + first + 32);
      }
      bool ok = true;
      if (lane == 0 && j >= kS) ok = tc::wait_bounded(&bars[kKEmpty0 + st], par, abort_flag, p.err, 10);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      uint8_t* kst = smem + C::kOffK + st * C::kKVBytes;
      if (lane == 0) mbar_arrive_expect_tx(&bars[kKFull0 + st], C::kKVBytes);
      for (int pi = 0; pi < ppt; ++pi) {
        const int r = __shfl_sync(0xffffffffu, cur, (first & 31) + pi);
        if (lane == 0) tc::tma_load_4d_w(kst + pi * page_bytes, &tm_kv, r, &bars[kKFull0 + st]);
      }
      if (lane == 0 && j >= kS) ok = tc::wait_bounded(&bars[kVEmpty0 + st], par, abort_flag, p.err, 11);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      uint8_t* vst = smem + C::kOffV + st * C::kKVBytes;
      if (lane == 0) mbar_arrive_expect_tx(&bars[kVFull0 + st], C::kKVBytes);
      for (int pi = 0; pi < ppt; ++pi) {
        const int r = __shfl_sync(0xffffffffu, cur, (first & 31) + pi);
        if (lane == 0) tc::tma_load_4d_w(vst + pi * page_bytes, &tm_kv, r + dv, &bars[kVFull0 + st]);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    // Both contractions take their M x K operand from TMEM (Q for S = Q K^T,
    // P for O += P V), so the tensor core reads only K and V from shared
    // memory.  S(j+1) runs while the softmax works on tile j; P(j) V follows
    // once P(j) is written.  tcgen05.mma of one thread execute in issue
    // order, so S(j+2) overwrites P(j) only after P(j) V has read it.
    if (lane == 0) {
      constexpr uint32_t idS = tc::idesc_bf16(kBM, C::kBN, false);
      constexpr uint32_t idO = tc::idesc_bf16(kBM, D, true);
      // K as the K-major B operand: 8-row groups kGroupBytes apart (SBO).
      const uint64_t dK = tc::sdesc_sw128(smem_u32(smem + C::kOffK), 16, C::kGroupBytes);
      // V as the MN-major B operand: 64-wide head-dim blocks 1024 bytes
      // apart (LBO), 8-row groups kGroupBytes apart (SBO).
      const uint64_t dV = tc::sdesc_sw128(smem_u32(smem + C::kOffV), 1024, C::kGroupBytes);
      // S = Q K^T: a 16-wide k step is 8 TMEM columns of Q, and 32 bytes
      // inside a 128-byte swizzle row of K (then the next 64-wide block).
      auto issue_s = [&](int j) -> bool {
        const int st = j % kS;
        if (!tc::wait_bounded(&bars[kKFull0 + st], (j / kS) & 1, abort_flag, p.err, 21)) return false;
        tc::fence_after_sync();
        const uint64_t b0 = dK + ((st * C::kKVBytes) >> 4);
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          tc::mma_bf16_ts(tmem + C::kTmemS + (j & 1) * C::kBN, tmem + C::kTmemQ + k * 8,
                          b0 + (((k >> 2) * 1024 + (k & 3) * 32) >> 4), idS, k > 0 ? 1u : 0u);
        if constexpr (PREC) {
#pragma unroll
          for (int k = 0; k < D / 16; ++k)
            tc::mma_bf16_ts(tmem + C::kTmemS + (j & 1) * C::kBN, tmem + C::kTmemQlo + k * 8,
                            b0 + (((k >> 2) * 1024 + (k & 3) * 32) >> 4), idS, 1u);
        }
        tc::mma_commit(&bars[kSFull0 + (j & 1)]);
        tc::mma_commit(&bars[kKEmpty0 + st]);
        return true;
      };
      bool ok = tc::wait_bounded(&bars[kQReady], 0, abort_flag, p.err, 20);
      if (ok) tc::fence_after_sync();
      ok = ok && issue_s(0);
      for (int j = 0; ok && j < nt; ++j) {  // j counts the range's tiles
        if (j + 1 < nt && !issue_s(j + 1)) break;
        const int st = j % kS;
        if (!tc::wait_bounded(&bars[kPFull0 + (j & 1)], (j >> 1) & 1, abort_flag, p.err, 22)) break;
        if (!tc::wait_bounded(&bars[kVFull0 + st], (j / kS) & 1, abort_flag, p.err, 23)) break;
        tc::fence_after_sync();
        // O += P V: a 16-token k step is 8 TMEM columns of P and two 8-row
        // groups of V.
        const uint64_t b0 = dV + ((st * C::kKVBytes) >> 4);
#pragma unroll
        for (int k = 0; k < C::kBN / 16; ++k)
          tc::mma_bf16_ts(tmem + C::kTmemO, tmem + C::kTmemS + (j & 1) * C::kBN + k * 8,
                          b0 + ((k * 2 * C::kGroupBytes) >> 4), idO, (j > 0 || k > 0) ? 1u : 0u);
        if constexpr (PREC) {
#pragma unroll
          for (int k = 0; k < C::kBN / 16; ++k)
            tc::mma_bf16_ts(tmem + C::kTmemO, tmem + C::kTmemS + (j & 1) * C::kBN + C::kBN / 2 + k * 8,
                            b0 + ((k * 2 * C::kGroupBytes) >> 4), idO, 1u);
        }
        tc::mma_commit(&bars[kODone0 + (j & 1)]);
        tc::mma_commit(&bars[kVEmpty0 + st]);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int row = threadIdx.x;  // 0..127 == TMEM lane
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const int row_pos = min(pos0 + row, last_pos);
    // Q row (bf16 pairs) into TMEM, every load in flight at once; rows past
    // the chunk are zero.  f32 queries are rounded to bf16 here (and with
    // split operands their remainders go to the second Q region).
    {
      const int64_t qoff = ((static_cast<int64_t>(q0) + tile * kBM + row) * p.hq + h) * D;
      uint4 v[D / 8];
      if (p.q_f32) {
        const float4* qrow = reinterpret_cast<const float4*>(static_cast<const float*>(p.q) + qoff);
        float4 f[D / 4];
#pragma unroll
        for (int i = 0; i < D / 4; ++i) f[i] = row < nrows ? qrow[i] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int i = 0; i < D / 8; ++i)
          v[i] = make_uint4(f2_to_bf2(f[2 * i].x, f[2 * i].y), f2_to_bf2(f[2 * i].z, f[2 * i].w),
                            f2_to_bf2(f[2 * i + 1].x, f[2 * i + 1].y), f2_to_bf2(f[2 * i + 1].z, f[2 * i + 1].w));
        if constexpr (PREC) {
#pragma unroll
          for (int c = 0; c < D / 64; ++c) {
            uint32_t r[32];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int e = c * 8 + i;
              r[4 * i] = bf2_residual(v[e].x, f[2 * e].x, f[2 * e].y);
              r[4 * i + 1] = bf2_residual(v[e].y, f[2 * e].z, f[2 * e].w);
              r[4 * i + 2] = bf2_residual(v[e].z, f[2 * e + 1].x, f[2 * e + 1].y);
              r[4 * i + 3] = bf2_residual(v[e].w, f[2 * e + 1].z, f[2 * e + 1].w);
            }
            tc::tmem_st32(lane_base + C::kTmemQlo + c * 32, r);
          }
        }
      } else {
        const uint4* qrow = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.q) + qoff);
#pragma unroll
        for (int i = 0; i < D / 8; ++i) v[i] = row < nrows ? qrow[i] : make_uint4(0u, 0u, 0u, 0u);
        if constexpr (PREC) {  // bf16 queries: no remainder
          uint32_t z[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) z[i] = 0u;
#pragma unroll
          for (int c = 0; c < D / 64; ++c) tc::tmem_st32(lane_base + C::kTmemQlo + c * 32, z);
        }
      }
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        uint32_t r[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          r[4 * i] = v[c * 8 + i].x;
          r[4 * i + 1] = v[c * 8 + i].y;
          r[4 * i + 2] = v[c * 8 + i].z;
          r[4 * i + 3] = v[c * 8 + i].w;
        }
        tc::tmem_st32(lane_base + C::kTmemQ + c * 32, r);
      }
      tc::tmem_st_wait();
      tc::fence_before_sync();
      tc::mbar_arrive(&bars[kQReady]);
    }
    float m_ref = -INFINITY, l_run = 0.0f;
    bool ok = true;
    for (int j = 0; j < nt; ++j) {  // j counts the range's tiles
      ok = softmax_tile<D, C::kBN, PREC>(lane_base, C::kTmemS + (j & 1) * C::kBN, C::kTmemO, (ja + j) * C::kBN, pos0,
                                   row_pos, p.qscale, m_ref, l_run, &bars[kSFull0 + (j & 1)], (j >> 1) & 1,
                                   &bars[kODone0 + ((j - 1) & 1)], ((j - 1) >> 1) & 1, &bars[kPFull0 + (j & 1)],
                                   abort_flag, p.err, 30);
      if (!ok) break;
    }
    // ---- epilogue: O / l (phantom key folded in), one row per thread.
    if (ok) ok = tc::wait_bounded(&bars[kODone0 + ((nt - 1) & 1)], ((nt - 1) >> 1) & 1, abort_flag, p.err, 32);
    tc::fence_after_sync();
    const bool valid = row < nrows;
    const int64_t orow = (static_cast<int64_t>(q0) + tile * kBM + row) * p.hq + h;
    auto store_chunk = [&](int c, const float* v, float inv) {
      if (valid) store_row_chunk(p, orow * D + c * 32, v, inv);
    };
    auto finish = [&](float m, float l) -> float { return row_inv_sum(p.phantom, m, l); };
    // Every softmax thread takes the same branch (k is per CTA; a failed
    // wait anywhere skips the merge's barriers in all four warps).
    const bool all_ok = !tc::named_sync_or(1, kBM, !ok);
    if (all_ok && k == 1) {
      const float inv = finish(m_ref, l_run);
      if (p.lse != nullptr && valid) p.lse[orow] = row_lse(p.phantom, m_ref, l_run);
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        tc::tmem_ld32(lane_base + C::kTmemO + c * 32, r);
        tc::tmem_ld_wait();
        store_chunk(c, reinterpret_cast<const float*>(r), inv);
      }
    } else if (all_ok) {
      // This piece's partial (O unnormalised, m, l), then a ticket; the last
      // piece to arrive merges all k in piece order.  Partials are laid out
      // [chunk][float4][row] so a warp's accesses are contiguous.
      const int64_t base = uid * kMaxPieces;
      float4* wo = reinterpret_cast<float4*>(p.ws_o);
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        tc::tmem_ld32(lane_base + C::kTmemO + c * 32, r);
        tc::tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 8; ++i)
          wo[(((base + piece) * (D / 32) + c) * 8 + i) * kBM + row] =
              make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]), __uint_as_float(r[4 * i + 2]),
                          __uint_as_float(r[4 * i + 3]));
      }
      p.ws_ml[((base + piece) * 2) * kBM + row] = m_ref;
      p.ws_ml[((base + piece) * 2 + 1) * kBM + row] = l_run;
      __threadfence();
      volatile int* last_s = reinterpret_cast<volatile int*>(smem + C::kOffMisc + 8);
      tc::named_sync(1, kBM);
      if (row == 0) *last_s = atomicAdd(&p.ws_cnt[uid], 1u) == static_cast<unsigned int>(k - 1) ? 1 : 0;
      tc::named_sync(1, kBM);
      if (*last_s) {
        __threadfence();
        float mi[kMaxPieces], li[kMaxPieces];
        float M = -INFINITY;
#pragma unroll
        for (int i = 0; i < kMaxPieces; ++i) {
          mi[i] = -INFINITY;
          li[i] = 0.0f;
          if (i < k) {
            mi[i] = i == piece ? m_ref : __ldcg(&p.ws_ml[((base + i) * 2) * kBM + row]);
            li[i] = i == piece ? l_run : __ldcg(&p.ws_ml[((base + i) * 2 + 1) * kBM + row]);
          }
          M = fmaxf(M, mi[i]);
        }
        float L = 0.0f;
#pragma unroll
        for (int i = 0; i < kMaxPieces; ++i) {
          mi[i] = mi[i] == -INFINITY ? 0.0f : exp2f(mi[i] - M);  // now the piece's weight
          L += li[i] * mi[i];
        }
        const float inv = finish(M, L);
        if (p.lse != nullptr && valid) p.lse[orow] = row_lse(p.phantom, M, L);
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t r[32];
          tc::tmem_ld32(lane_base + C::kTmemO + c * 32, r);
          tc::tmem_ld_wait();
          float acc[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) acc[e] = 0.0f;
#pragma unroll
          for (int i = 0; i < kMaxPieces; ++i) {
            const float a = mi[i];
            if (i >= k) {
            } else if (i == piece) {
#pragma unroll
              for (int e = 0; e < 32; ++e) acc[e] = fmaf(__uint_as_float(r[e]), a, acc[e]);
            } else {
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                const float4 v = __ldcg(&wo[(((base + i) * (D / 32) + c) * 8 + q) * kBM + row]);
                acc[4 * q] = fmaf(v.x, a, acc[4 * q]);
                acc[4 * q + 1] = fmaf(v.y, a, acc[4 * q + 1]);
                acc[4 * q + 2] = fmaf(v.z, a, acc[4 * q + 2]);
                acc[4 * q + 3] = fmaf(v.w, a, acc[4 * q + 3]);
              }
            }
          }
          store_chunk(c, acc, inv);
        }
        if (row == 0) p.ws_cnt[uid] = 0u;  // ready for the next call on this workspace
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ------------------------------------------------ two query tiles per CTA
// For head_dim 64 and 128 a CTA can hold two 128-row query tiles of one
// (head, sequence): S and O of both fit the 512 TMEM columns once Q is read
// from shared memory instead of TMEM.  Each K/V tile then serves 256 query
// rows, halving the L2 -> SM traffic per FLOP, and the two softmax
// warpgroups alternate with the tensor core: while one works on its S, the
// MMA thread runs the other's P V and next S.
//   warps 0-3  softmax of query tile A (rows 2 t .. of the pair t), warps
//              4-7 of tile B (the next 128 rows, when the chunk has them);
//              each first writes its Q tile to shared memory, 128B-swizzled.
//   warp 8     producer (as in the one-tile kernel).
//   warp 9     MMA issuer: S_A(0), S_B(0), then per kv tile j: P_A(j) V,
//              S_A(j+1), P_B(j) V, S_B(j+1).
// 320 threads: three warps share an SM sub-partition, so a thread gets up
// to 168 registers.
constexpr int kPairThreads = 320;

template <int D>
struct QCfg {
  static constexpr int kBN = 128;                      // kv tokens per tile
  static constexpr int kDB = D / 64;
  static constexpr int kStages = D == 128 ? 2 : 3;     // K/V ring depth
  static constexpr int kKVBytes = kBN * D * 2;
  static constexpr int kQBytes = kBM * D * 2;          // [D/64 blocks][128 rows][128 B]
  static constexpr int kGroupBytes = kDB * 1024;
  static constexpr int kOffQ = 0;                      // [2][kQBytes]
  static constexpr int kOffK = 2 * kQBytes;
  static constexpr int kOffV = kOffK + kStages * kKVBytes;
  static constexpr int kOffBar = kOffV + kStages * kKVBytes;
  static constexpr int kOffMisc = kOffBar + 24 * 8;
  static constexpr int kSmem = kOffMisc + 64 + 1024;
  static constexpr int kTmemS = 0;                     // S of tile X at X * kBN
  static constexpr int kTmemO = 2 * kBN;               // O of tile X at kTmemO + X * D
  static constexpr int kTmemCols = 512;
  static_assert(kTmemO + 2 * D <= kTmemCols, "TMEM budget");
  static_assert(kSmem <= 227 * 1024, "shared memory");
};

enum PairBar {
  qQReady0 = 0,   // [2] Q of tile X in shared memory (128 threads each)
  qKFull0 = 2,    // [3]
  qVFull0 = 5,    // [3]
  qKEmpty0 = 8,   // [3] S of both tiles done with the stage's K
  qVEmpty0 = 11,  // [3] P V of both tiles done with the stage's V
  qSFull0 = 14,   // [2] S of tile X holds kv tile j's scores
  qPFull0 = 16,   // [2] P of tile X written (128 threads each)
  qODone0 = 18,   // [2] P V of tile X's kv tile j done
  qNumBars = 20
};

template <int D>
__global__ void __launch_bounds__(kPairThreads, 1)
    paged_prefill_pair_kernel(const __grid_constant__ CUtensorMap tm_kv, const __grid_constant__ PrefillParams p) {
  using C = QCfg<D>;
  constexpr int kS = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int pair = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
  const int q0 = p.qo_indptr[s];
  const int q_len = p.qo_indptr[s + 1] - q0;
  const int t0 = 2 * pair;  // query tile A; B = t0 + 1
  if (t0 * kBM >= q_len) return;
  const int kv_beg = p.kv_indptr[s];
  const int npages = p.kv_indptr[s + 1] - kv_beg;
  int kv_len = p.seq_lens[s];
  if (kv_len < q_len || kv_len > npages * p.ps) {
    if (pair == 0 && h == 0 && threadIdx.x == 0) record_error(p.err, kDevErrBadSeqLen, s);
    kv_len = max(q_len, min(kv_len, npages * p.ps));
    if (kv_len > npages * p.ps) return;  // not even the chunk fits its pages
  }
  const bool has_b = (t0 + 1) * kBM < q_len;
  const int pos0a = kv_len - q_len + t0 * kBM;  // position of tile A's row 0
  const int nrows_a = min(kBM, q_len - t0 * kBM);
  const int nrows_b = has_b ? min(kBM, q_len - (t0 + 1) * kBM) : 0;
  const int n_a = (pos0a + nrows_a - 1) / C::kBN + 1;                   // kv tiles tile A sees
  const int n_b = has_b ? (pos0a + kBM + nrows_b - 1) / C::kBN + 1 : 0;  // >= n_a
  const int n = max(n_a, n_b);
  const int g = h / (p.hq / p.hkv);

  if (threadIdx.x == 0) {
    for (int i = 0; i < qNumBars; ++i)
      mbar_init(&bars[i], (i == qQReady0 || i == qQReady0 + 1 || i == qPFull0 || i == qPFull0 + 1) ? kBM : 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(tmem_base_s, C::kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_base_s;

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    // As in the one-tile kernel: one 4-D box per (page, kv head), page ids
    // fetched 32 at a time one window ahead, K refilled once S of both
    // query tiles is done with the stage, V once both P V are.
    const int ppt = C::kBN / p.ps;
    const int lim = min(npages, n * ppt) - 1;
    auto fetch = [&](int first) -> int { return p.kv_indices[kv_beg + min(first + lane, lim)]; };
    auto to_row = [&](int page) -> int {
      if (page < 0 || page >= p.num_pages) {
        record_error(p.err, kDevErrBadPage, s);
        page = 0;
      }
      return static_cast<int>((p.row_k + (static_cast<int64_t>(page) * p.hkv + g) * p.ps) >> 3);
    };
    if (lane == 0) tc::prefetch_tmap(&tm_kv);
    const int page_bytes = p.ps * D * 2;
    const int dv = static_cast<int>((p.row_v - p.row_k) >> 3);
    int cur = to_row(fetch(0));
    int nxt = fetch(32);
    for (int j = 0; j < n; ++j) {
      const int st = j % kS;
      const uint32_t par = ((j / kS) - 1) & 1;
      const int first = j * ppt;
      if (j > 0 && (first & 31) == 0) {
        cur = to_row(nxt);
        nxt = fetch(first + 32);
      }
      bool ok = true;
      if (lane == 0 && j >= kS) ok = tc::wait_bounded(&bars[qKEmpty0 + st], par, abort_flag, p.err, 50);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      uint8_t* kst = smem + C::kOffK + st * C::kKVBytes;
      if (lane == 0) mbar_arrive_expect_tx(&bars[qKFull0 + st], C::kKVBytes);
      for (int pi = 0; pi < ppt; ++pi) {
        const int r = __shfl_sync(0xffffffffu, cur, (first & 31) + pi);
        if (lane == 0) tc::tma_load_4d_w(kst + pi * page_bytes, &tm_kv, r, &bars[qKFull0 + st]);
      }
      if (lane == 0 && j >= kS) ok = tc::wait_bounded(&bars[qVEmpty0 + st], par, abort_flag, p.err, 51);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      uint8_t* vst = smem + C::kOffV + st * C::kKVBytes;
      if (lane == 0) mbar_arrive_expect_tx(&bars[qVFull0 + st], C::kKVBytes);
      for (int pi = 0; pi < ppt; ++pi) {
        const int r = __shfl_sync(0xffffffffu, cur, (first & 31) + pi);
        if (lane == 0) tc::tma_load_4d_w(vst + pi * page_bytes, &tm_kv, r + dv, &bars[qVFull0 + st]);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    // S_X = Q_X K^T with both operands in shared memory (Q block-major: 64
    // columns x 128 rows per 16 KB block at head_dim 128); O_X += P_X V with
    // P_X from TMEM.  One thread's tcgen05.mma execute in issue order, so
    // S_X(j+1), issued after P_X(j) V, overwrites P_X(j) only once it is read.
    if (lane == 0) {
      constexpr uint32_t idS = tc::idesc_bf16(kBM, C::kBN, false);
      constexpr uint32_t idO = tc::idesc_bf16(kBM, D, true);
      const uint64_t dQ = tc::sdesc_sw128(smem_u32(smem + C::kOffQ), 16, 1024);
      const uint64_t dK = tc::sdesc_sw128(smem_u32(smem + C::kOffK), 16, C::kGroupBytes);
      const uint64_t dV = tc::sdesc_sw128(smem_u32(smem + C::kOffV), 1024, C::kGroupBytes);
      auto issue_s = [&](int x, int j) -> bool {
        const int st = j % kS;
        if (!tc::wait_bounded(&bars[qKFull0 + st], (j / kS) & 1, abort_flag, p.err, 60)) return false;
        tc::fence_after_sync();
        const uint64_t a0 = dQ + ((x * C::kQBytes) >> 4);
        const uint64_t b0 = dK + ((st * C::kKVBytes) >> 4);
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          tc::mma_bf16(tmem + C::kTmemS + x * C::kBN, a0 + (((k >> 2) * (kBM * 128) + (k & 3) * 32) >> 4),
                       b0 + (((k >> 2) * 1024 + (k & 3) * 32) >> 4), idS, k > 0 ? 1u : 0u);
        tc::mma_commit(&bars[qSFull0 + x]);
        return true;
      };
      auto issue_pv = [&](int x, int j) -> bool {
        const int st = j % kS;
        if (!tc::wait_bounded(&bars[qPFull0 + x], j & 1, abort_flag, p.err, 61)) return false;
        if (!tc::wait_bounded(&bars[qVFull0 + st], (j / kS) & 1, abort_flag, p.err, 62)) return false;
        tc::fence_after_sync();
        const uint64_t b0 = dV + ((st * C::kKVBytes) >> 4);
#pragma unroll
        for (int k = 0; k < C::kBN / 16; ++k)
          tc::mma_bf16_ts(tmem + C::kTmemO + x * D, tmem + C::kTmemS + x * C::kBN + k * 8,
                          b0 + ((k * 2 * C::kGroupBytes) >> 4), idO, (j > 0 || k > 0) ? 1u : 0u);
        tc::mma_commit(&bars[qODone0 + x]);
        return true;
      };
      bool ok = tc::wait_bounded(&bars[qQReady0], 0, abort_flag, p.err, 63);
      if (ok && has_b) ok = tc::wait_bounded(&bars[qQReady0 + 1], 0, abort_flag, p.err, 63);
      if (ok) tc::fence_after_sync();
      ok = ok && issue_s(0, 0) && (!has_b || issue_s(1, 0));
      if (ok) tc::mma_commit(&bars[qKEmpty0]);
      for (int j = 0; ok && j < n; ++j) {
        if (j < n_a) {
          ok = issue_pv(0, j) && (j + 1 >= n_a || issue_s(0, j + 1));
          if (!ok) break;
        }
        if (j < n_b) {
          ok = issue_pv(1, j) && (j + 1 >= n_b || issue_s(1, j + 1));
          if (!ok) break;
        }
        tc::mma_commit(&bars[qVEmpty0 + j % kS]);
        if (j + 1 < n) tc::mma_commit(&bars[qKEmpty0 + (j + 1) % kS]);
      }
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------ softmax
    const int x = warp >> 2;  // query tile of this warpgroup
    if (x == 0 || has_b) {
      const int row = threadIdx.x & (kBM - 1);  // == TMEM lane
      const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
      const int nrows = x ? nrows_b : nrows_a;
      const int pos0 = pos0a + x * kBM;
      const int last_pos = pos0 + nrows - 1;
      const int nx = x ? n_b : n_a;
      const int row_pos = min(pos0 + row, last_pos);
      const int64_t qrow0 = static_cast<int64_t>(q0) + (t0 + x) * kBM + row;
      {
        // Q row into shared memory: 16-byte chunk c of the row goes to block
        // c / 8, chunk (c % 8) ^ (row % 8) of the row's 128 bytes (the
        // 128-byte swizzle the descriptor names); rows past the chunk are zero.
        const uint4* qrow =
            reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.q) + (qrow0 * p.hq + h) * D);
        uint8_t* qs = smem + C::kOffQ + x * C::kQBytes + row * 128;
#pragma unroll
        for (int b = 0; b < D / 64; ++b) {  // one 64-column block (8 chunks) at a time
          uint4 v[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = row < nrows ? qrow[b * 8 + i] : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
          for (int c = 0; c < 8; ++c)
            *reinterpret_cast<uint4*>(qs + b * (kBM * 128) + ((c ^ (row & 7)) << 4)) = v[c];
        }
        fence_proxy_async_shared();
        tc::mbar_arrive(&bars[qQReady0 + x]);
      }
      float m_ref = -INFINITY, l_run = 0.0f;
      bool ok = true;
      for (int j = 0; j < nx; ++j) {
        ok = softmax_tile<D, C::kBN, false>(lane_base, C::kTmemS + x * C::kBN, C::kTmemO + x * D, j * C::kBN, pos0, row_pos,
                                     p.qscale, m_ref, l_run, &bars[qSFull0 + x], j & 1, &bars[qODone0 + x],
                                     (j - 1) & 1, &bars[qPFull0 + x], abort_flag, p.err, 70);
        if (!ok) break;
      }
      if (ok) ok = tc::wait_bounded(&bars[qODone0 + x], (nx - 1) & 1, abort_flag, p.err, 72);
      tc::fence_after_sync();
      if (!tc::named_sync_or(1 + x, kBM, !ok)) {
        const float inv = row_inv_sum(p.phantom, m_ref, l_run);
        const int64_t elem0 = (qrow0 * p.hq + h) * D;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t r[32];
          tc::tmem_ld32(lane_base + C::kTmemO + x * D + c * 32, r);
          tc::tmem_ld_wait();
          if (row < nrows) store_row_chunk(p, elem0 + c * 32, reinterpret_cast<const float*>(r), inv);
        }
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, C::kTmemCols);
  }
}

// --------------------------------------------------------------- host side

template <int D, bool PREC = false>
int launch_prefill(const CUtensorMap& tkv, const PrefillParams& prm, int n_tiles, int n_seqs,
                   cudaStream_t stream) {
  using C = PCfg<D>;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    MTN_CUDA_TRY(cudaFuncSetAttribute(paged_prefill_kernel<D, PREC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      C::kSmem),
                 "cudaFuncSetAttribute(prefill)");
    configured[dev] = true;
  }
  dim3 grid(n_tiles, prm.hq, prm.split ? n_seqs * kMaxPieces : n_seqs);
  paged_prefill_kernel<D, PREC><<<grid, kThreads, C::kSmem, stream>>>(tkv, prm);
  return check_launch("paged_prefill_kernel");
}

template <int D>
int launch_prefill_pair(const CUtensorMap& tkv, const PrefillParams& prm, int n_tiles, int n_seqs,
                        cudaStream_t stream) {
  using C = QCfg<D>;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    MTN_CUDA_TRY(cudaFuncSetAttribute(paged_prefill_pair_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      C::kSmem),
                 "cudaFuncSetAttribute(prefill pair)");
    configured[dev] = true;
  }
  dim3 grid((n_tiles + 1) / 2, prm.hq, n_seqs);
  paged_prefill_pair_kernel<D><<<grid, kPairThreads, C::kSmem, stream>>>(tkv, prm);
  return check_launch("paged_prefill_pair_kernel");
}

// Workspace of the split: counters, then (m, l) rows, then O partials.
struct SplitLayout {
  int64_t units = 0;
  size_t off_ml = 0, off_o = 0, bytes = 0;
};

SplitLayout split_layout(int32_t n_seqs, int64_t total_q, int32_t num_q_heads, int32_t head_dim) {
  SplitLayout w;
  if (n_seqs <= 0 || total_q <= 0 || num_q_heads <= 0 || head_dim <= 0) return w;
  const int64_t units = (total_q / kBM + n_seqs) * num_q_heads;
  if (units > kSplitMaxUnits) return w;  // enough units to fill the GPU: no split
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  const size_t slots = static_cast<size_t>(units) * kMaxPieces;
  w.units = units;
  w.off_ml = up(static_cast<size_t>(units) * 4);
  w.off_o = w.off_ml + up(slots * 2 * kBM * 4);
  w.bytes = w.off_o + slots * kBM * static_cast<size_t>(head_dim) * 4;
  return w;
}

}  // namespace
}  // namespace mtn

using mtn::set_error;

extern "C" {

size_t mtn_paged_prefill_workspace_bytes(int32_t n_seqs, int64_t total_q, int32_t num_q_heads, int32_t num_kv_heads,
                                         int32_t head_dim) {
  (void)num_kv_heads;
  return mtn::split_layout(n_seqs, total_q, num_q_heads, head_dim).bytes;
}

int mtn_paged_prefill(const mtn_kv_layout* pool, int32_t layer, const void* q, int32_t q_dtype, void* o,
                      int32_t o_dtype,
                      int32_t n_seqs, int64_t total_q, int32_t num_q_heads, const int32_t* qo_indptr,
                      const int32_t* kv_indptr, const int32_t* kv_indices, const int32_t* seq_lens, int32_t max_q_len,
                      float scale, uint32_t flags, void* workspace, size_t workspace_bytes, void* stream) {
  return mtn::paged_prefill_impl(pool, layer, q, q_dtype, o, o_dtype, n_seqs, total_q, num_q_heads, qo_indptr,
                                 kv_indptr, kv_indices, seq_lens, max_q_len, scale, flags, workspace, workspace_bytes,
                                 stream, 0, nullptr, 0);
}

}  // extern "C"

namespace mtn {

int paged_prefill_impl(const mtn_kv_layout* pool, int32_t layer, const void* q, int32_t q_dtype, void* o,
                       int32_t o_dtype, int32_t n_seqs, int64_t total_q, int32_t num_q_heads,
                       const int32_t* qo_indptr, const int32_t* kv_indptr, const int32_t* kv_indices,
                       const int32_t* seq_lens, int32_t max_q_len, float scale, uint32_t flags, void* workspace,
                       size_t workspace_bytes, void* stream, int noncausal, float* lse, int nc_pages) {
  // noncausal: one pseudo-sequence (n_seqs must be 1) of total_q query rows
  // over the pages kv_indices[0 .. nc_pages); qo_indptr, kv_indptr and
  // seq_lens are not read.
  int st = mtn::validate_layout(pool, layer, "mtn_paged_prefill");
  if (st != MTN_OK) return st;
  MTN_CHECK_ARG(n_seqs >= 0 && n_seqs <= 65535, "mtn_paged_prefill: n_seqs %d outside [0, 65535]", n_seqs);
  MTN_CHECK_ARG(total_q >= 0 && total_q < (int64_t(1) << 31), "mtn_paged_prefill: bad total_q");
  if (n_seqs == 0 || total_q == 0) return MTN_OK;
  MTN_CHECK_ARG(q && o && kv_indices && (noncausal || (qo_indptr && kv_indptr && seq_lens)),
                "mtn_paged_prefill: null pointer");
  MTN_CHECK_ARG(!noncausal || (n_seqs == 1 && nc_pages > 0), "mtn_paged_prefill: bad non-causal launch");
  MTN_CHECK_ARG(q_dtype == MTN_DTYPE_BF16 || q_dtype == MTN_DTYPE_F32, "mtn_paged_prefill: bad q dtype");
  MTN_CHECK_ARG(o_dtype == MTN_DTYPE_BF16 || o_dtype == MTN_DTYPE_F32, "mtn_paged_prefill: bad o dtype");
  MTN_CHECK_ARG(num_q_heads > 0 && num_q_heads <= 65535 && num_q_heads % pool->num_kv_heads == 0,
                "mtn_paged_prefill: %d query heads not a multiple of %d kv heads", num_q_heads, pool->num_kv_heads);
  MTN_CHECK_ARG(max_q_len > 0, "mtn_paged_prefill: max_q_len must be positive");
  const int D = pool->head_dim;
  const int bn = D <= 128 ? 128 : 64;
  MTN_CHECK_ARG(pool->page_size <= bn && bn % pool->page_size == 0 && pool->page_size % 8 == 0,
                "mtn_paged_prefill: page_size %d must be a multiple of 8 dividing %d", pool->page_size, bn);
  MTN_CHECK_ARG((reinterpret_cast<uintptr_t>(q) & 15) == 0 && (reinterpret_cast<uintptr_t>(o) & 15) == 0,
                "mtn_paged_prefill: q/o must be 16-byte aligned");
  const bool prec = (flags & MTN_ATTN_SPLIT_BF16) != 0;
  MTN_CHECK_ARG(!prec || D <= 128, "mtn_paged_prefill: MTN_ATTN_SPLIT_BF16 needs head_dim <= 128 (got %d)", D);
  CUtensorMap tkv;
  st = mtn::pool_tensor_map_paged(pool, &tkv);
  if (st != MTN_OK) return st;
  mtn::PrefillParams prm{};
  prm.q = q;
  prm.q_f32 = q_dtype == MTN_DTYPE_F32;
  prm.qo_indptr = qo_indptr;
  prm.kv_indptr = kv_indptr;
  prm.kv_indices = kv_indices;
  prm.seq_lens = seq_lens;
  prm.o = o;
  prm.o_f32 = o_dtype == MTN_DTYPE_F32;
  prm.hq = num_q_heads;
  prm.hkv = pool->num_kv_heads;
  prm.ps = pool->page_size;
  prm.num_pages = pool->num_pages;
  const int64_t rows_per_block = pool->num_pages * pool->num_kv_heads * pool->page_size;
  prm.row_k = (static_cast<int64_t>(layer) * 2 + 0) * rows_per_block;
  prm.row_v = (static_cast<int64_t>(layer) * 2 + 1) * rows_per_block;
  prm.qscale = scale * mtn::kLog2e;
  prm.phantom = (flags & MTN_ATTN_PHANTOM_ZERO_SLOT) ? 1 : 0;
  prm.err = mtn::device_error_ptr();
  prm.noncausal = noncausal;
  prm.lse = lse;
  prm.nc_q_len = static_cast<int>(total_q);
  prm.nc_pages = nc_pages;
  const int n_tiles = (max_q_len + mtn::kBM - 1) / mtn::kBM;
  MTN_CHECK_ARG(n_tiles <= 65535 * 32, "mtn_paged_prefill: max_q_len too large");
  // Launches whose units (bounded by (total_q / 128 + n_seqs) x heads) leave
  // a quarter or more of the SMs idle split long units across more CTAs when
  // the workspace is there; otherwise they run unsplit (same results).
  const mtn::SplitLayout wl = mtn::split_layout(n_seqs, total_q, num_q_heads, D);
  if (wl.bytes > 0 && wl.units * 4 <= 3 * static_cast<int64_t>(mtn::sm_count()) && workspace != nullptr &&
      workspace_bytes >= wl.bytes && (reinterpret_cast<uintptr_t>(workspace) & 255) == 0) {
    uint8_t* w = static_cast<uint8_t*>(workspace);
    prm.split = 1;
    prm.split_target = mtn::sm_count();
    prm.n_seqs = n_seqs;
    prm.max_units = wl.units;
    prm.ws_cnt = reinterpret_cast<unsigned int*>(w);
    prm.ws_ml = reinterpret_cast<float*>(w + wl.off_ml);
    prm.ws_o = reinterpret_cast<float*>(w + wl.off_o);
  }
  auto s = static_cast<cudaStream_t>(stream);
  if (prec) {
    return D == 64 ? mtn::launch_prefill<64, true>(tkv, prm, n_tiles, n_seqs, s)
                   : mtn::launch_prefill<128, true>(tkv, prm, n_tiles, n_seqs, s);
  }
  // Many query tiles (at least two per SM): two tiles per CTA at head_dim
  // <= 128, sharing every K/V tile (bf16 queries).
  if (!prm.split && !noncausal && lse == nullptr && D <= 128 && !prm.q_f32 && !(flags & MTN_ATTN_PREFILL_ONE_TILE) &&
      (total_q / mtn::kBM) * num_q_heads >= 2 * static_cast<int64_t>(mtn::sm_count())) {
    return D == 64 ? mtn::launch_prefill_pair<64>(tkv, prm, n_tiles, n_seqs, s)
                   : mtn::launch_prefill_pair<128>(tkv, prm, n_tiles, n_seqs, s);
  }
  switch (D) {
    case 64: return mtn::launch_prefill<64>(tkv, prm, n_tiles, n_seqs, s);
    case 128: return mtn::launch_prefill<128>(tkv, prm, n_tiles, n_seqs, s);
    default: return mtn::launch_prefill<256>(tkv, prm, n_tiles, n_seqs, s);
  }
}

}  // namespace mtn
