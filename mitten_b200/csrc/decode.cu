// Paged GQA/MQA decode attention for sm_100a (one query token per sequence).
//
// Replaces the decode-step attention of qwen model.rs:394-416: GQA head
// mapping h -> h / n_rep (model.rs:398-408), scores q.k * scale
// (model.rs:298, 413), softmax over every key including the reference's
// all-zero first row (model.rs:207-220, flag MTN_ATTN_PHANTOM_ZERO_SLOT),
// output P.V (model.rs:416).  One query token sees every key, so
// generate_causal_mask (model.rs:542-555) masks nothing here.
//
// Design.  The step is HBM-bound (every K/V byte is read once) but at GQA
// n_rep = 7 the arithmetic is 3.5 FMA per byte, more than the CUDA cores can
// issue at HBM speed, so both contractions run on the tensor cores with the
// n_rep query heads of one KV head as the narrow N dimension:
//   S^T[128 tokens][16] = K_tile[128][D] . Q^T            (tcgen05, M=128, N=16)
//   O^T[D][16]         += V_tile^T[D][128] . P^T[128][16] (tcgen05, M=D (64|128), N=16)
// grid = (split, kv head, sequence); a CTA owns `pages_per_split` pages of
// one sequence for one KV head.  6 warps:
//   warps 0-3  softmax: TMEM lane = token; online softmax in the exp2 domain
//              with a CTA-wide running max per query head, P^T (bf16) written
//              to shared memory, O^T rescaled in TMEM, epilogue.
//   warp 4     TMA producer: each page of each 128-token tile is one 2-D box
//              (page_size rows x 64 columns, 128B swizzle) straight from the
//              block table into a STAGES-deep ring.
//   warp 5     MMA issuer (one thread), completion through tcgen05.commit.
// Splits of one sequence write (m, l, O) partials to the workspace; the last
// CTA to arrive (atomic ticket, no spinning) merges them in split order, so
// the result does not depend on CTA scheduling.  Every wait is bounded.
#include <algorithm>
#include <cfloat>

#include "common.cuh"
#include "tc.cuh"
#include "tmaps.hpp"

namespace mtn {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kTile = 128;    // tokens per tile = MMA1 M = TMEM lanes
constexpr int kThreads = 192;
constexpr int kN = 16;        // query heads per KV head, padded (MMA N)

struct DecodeParams {
  int64_t num_pages;
  int64_t row_k;  // pool-view row of (layer K, page 0, head 0, token 0)
  int64_t row_v;
  int hkv;
  int ps;
  int hq;
  const void* q;
  void* o;
  int q_f32;
  int o_f32;
  const int32_t* kv_indptr;
  const int32_t* kv_indices;
  const int32_t* seq_lens;
  int pages_per_split;
  int max_splits;
  float qscale;  // scale * log2(e)
  int phantom;
  float* ws_o;           // [n_seqs][hq][max_splits][D]
  float* ws_ml;          // [n_seqs][hq][max_splits][2]
  unsigned int* ws_cnt;  // [n_seqs][hkv]
  int* err;
};

template <int D>
struct DCfg {
  static constexpr int kDB = D / 64;                       // 64-wide head-dim blocks
  static constexpr int kStages = D == 256 ? 1 : 2;
  static constexpr int kQBytes = kN * D * 2;               // Q^T operand: 16 rows x D
  static constexpr int kKVBytes = kTile * D * 2;           // one of K or V per stage
  static constexpr int kPBytes = kN * kTile * 2;           // P^T operand: 16 rows x 128 tokens
  static constexpr int kMaxSplitPages = 256;               // page ids staged per CTA
  // Small state first, then the 1 KiB-aligned operand area.
  static constexpr int kOffBar = 0;                        // 16 mbarriers
  static constexpr int kOffMisc = kOffBar + 16 * 8;        // tmem base, abort flag, last-CTA flag
  static constexpr int kOffRed = kOffMisc + 64;            // [2][4][16] maxima, [4][16] sums, [2] flags
  static constexpr int kOffIdx = kOffRed + (2 * 4 * kN + 4 * kN + 16) * 4;
  static constexpr int kSmallBytes = kOffIdx + kMaxSplitPages * 4;
  static constexpr int kOffQ = 0;                          // relative to the aligned operand area
  static constexpr int kOffK = kOffQ + kQBytes;
  static constexpr int kOffV = kOffK + kStages * kKVBytes;
  static constexpr int kOffP = kOffV + kStages * kKVBytes;
  static constexpr int kBigBytes = kOffP + kPBytes;
  static constexpr int kSmem = kSmallBytes + 1023 + kBigBytes;
  static constexpr int kMO = D == 64 ? 64 : 128;           // MMA2 M
  static constexpr int kTmemS = 0;                          // 2 x 16 columns (double-buffered S^T)
  static constexpr int kTmemO = 32;                         // 16 (D <= 128) or 32 (D = 256) columns
  static constexpr int kTmemCols = 64;
  static_assert(kOffK % 1024 == 0 && kOffV % 1024 == 0 && kOffP % 1024 == 0, "swizzle atoms need 1 KiB alignment");
};

// Lazy rescaling: P is exponentiated against a CTA-wide reference max that
// only moves when a tile's max exceeds it by more than 2^kRescaleLog2, so
// P <= 2^8 (exact in bf16 range) and O^T in TMEM is rarely touched.
constexpr float kRescaleLog2 = 8.0f;

enum Bar { kKVFull0 = 0, kKVFull1 = 1, kKVEmpty0 = 2, kKVEmpty1 = 3, kSFull0 = 4, kSFull1 = 5, kPFull = 6,
           kODone = 7 };

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

template <int D, int NREP>
__global__ void __launch_bounds__(kThreads, D == 64 ? 3 : 1)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tm_kv, const __grid_constant__ DecodeParams p) {
  using C = DCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw + C::kOffBar);
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(smem_raw + C::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem_raw + C::kOffMisc + 4);
  volatile int* last_flag = reinterpret_cast<volatile int*>(smem_raw + C::kOffMisc + 8);
  float* red_max = reinterpret_cast<float*>(smem_raw + C::kOffRed);  // [2][4][16]
  float* red_sum = red_max + 2 * 4 * kN;                             // [4][16]
  int* idx_s = reinterpret_cast<int*>(smem_raw + C::kOffIdx);        // this split's page ids
  uint8_t* big = smem_raw + C::kSmallBytes;
  big += (1024 - (smem_u32(big) & 1023)) & 1023;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split = blockIdx.x, g = blockIdx.y, s = blockIdx.z;

  const int pbeg = p.kv_indptr[s];
  const int ntab = p.kv_indptr[s + 1] - pbeg;
  int seq_len = p.seq_lens[s];
  if (seq_len < 0 || seq_len > ntab * p.ps) {
    if (split == 0 && g == 0 && threadIdx.x == 0) record_error(p.err, kDevErrBadSeqLen, s);
    seq_len = min(max(seq_len, 0), ntab * p.ps);
  }
  int npages = (seq_len + p.ps - 1) / p.ps;
  if (npages > p.max_splits * p.pages_per_split) {
    // More pages than max_pages_per_seq promised: the grid and the workspace
    // only cover max_splits splits, so attend to the covered prefix only.
    if (split == 0 && g == 0 && threadIdx.x == 0) record_error(p.err, kDevErrBadSeqLen, s);
    npages = p.max_splits * p.pages_per_split;
    seq_len = npages * p.ps;
  }
  const int n_splits = max(1, (npages + p.pages_per_split - 1) / p.pages_per_split);
  if (split >= n_splits) return;
  const int pg0 = split * p.pages_per_split;
  const int pg1 = min(npages, pg0 + p.pages_per_split);
  const int tok_begin = pg0 * p.ps;
  const int ntok = max(0, min(seq_len, pg1 * p.ps) - tok_begin);
  const int ntiles = (ntok + kTile - 1) / kTile;
  const int tile_pages = kTile / p.ps;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 8; ++i) mbar_init(&bars[i], i == kPFull ? 128 : 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    // Stage the split's page ids once (one coalesced round trip), then every
    // tile's boxes are issued by tile_pages lanes in parallel.
    for (int i = lane; i < pg1 - pg0; i += 32) {
      int64_t page = p.kv_indices[pbeg + pg0 + i];
      if (page < 0 || page >= p.num_pages) {
        record_error(p.err, kDevErrBadPage, s);
        page = 0;
      }
      idx_s[i] = static_cast<int>(page);
    }
    __syncwarp();
    if (lane == 0) tc::prefetch_tmap(&tm_kv);
    for (int j = 0; j < ntiles; ++j) {
      const int st = j % C::kStages;
      if (j >= C::kStages) {
        bool free_ok = true;
        if (lane == 0) free_ok = tc::wait_bounded(&bars[kKVEmpty0 + st], ((j / C::kStages) - 1) & 1, abort_flag, p.err, 10);
        if (!__shfl_sync(0xffffffffu, free_ok, 0)) break;  // warp-uniform
      }
      if (lane == 0) mbar_arrive_expect_tx(&bars[kKVFull0 + st], 2 * C::kKVBytes);
      __syncwarp();
      if (lane < tile_pages) {
        // Past the split's last page: reload that page (finite data, masked).
        const int pi = lane;
        const int64_t page = idx_s[min(j * tile_pages + pi, pg1 - pg0 - 1)];
        const int64_t rk = p.row_k + (page * p.hkv + g) * p.ps;
        const int64_t rv = p.row_v + (page * p.hkv + g) * p.ps;
        uint8_t* kst = big + C::kOffK + st * C::kKVBytes;
        uint8_t* vst = big + C::kOffV + st * C::kKVBytes;
#pragma unroll
        for (int b = 0; b < C::kDB; ++b) {
          const int off = b * kTile * 128 + pi * p.ps * 128;
          tc::tma_load_2d(kst + off, &tm_kv, b * 64, static_cast<int>(rk), &bars[kKVFull0 + st]);
          tc::tma_load_2d(vst + off, &tm_kv, b * 64, static_cast<int>(rv), &bars[kKVFull0 + st]);
        }
      }
    }
  } else {
    // Everyone else: TMEM, the Q^T operand (16 rows, rows >= NREP zero, 128B
    // swizzled K-major) and a zeroed P^T operand (rows >= NREP stay zero),
    // overlapping the producer's first loads.
    if (warp == 0) {
      tc::tmem_alloc(tmem_base_s, C::kTmemCols);
      tc::tmem_relinquish();
    }
    const int tid = warp == 5 ? 128 + lane : threadIdx.x;  // 0..159
    uint8_t* q_s = big + C::kOffQ;
    const int64_t qrow0 = static_cast<int64_t>(s) * p.hq + g * NREP;
    for (int e = tid; e < kN * (D / 8); e += 160) {
      const int r = e / (D / 8), c = e - r * (D / 8);
      const int b = c >> 3, cc = c & 7;
      uint4 w = make_uint4(0u, 0u, 0u, 0u);
      if (r < NREP) {
        const int64_t off = (qrow0 + r) * D + c * 8;
        if (p.q_f32) {
          const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(p.q) + off);
          const float4 bb = *(reinterpret_cast<const float4*>(static_cast<const float*>(p.q) + off) + 1);
          w = make_uint4(f2_to_bf2(a.x, a.y), f2_to_bf2(a.z, a.w), f2_to_bf2(bb.x, bb.y), f2_to_bf2(bb.z, bb.w));
        } else {
          w = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.q) + off);
        }
      }
      *reinterpret_cast<uint4*>(q_s + b * (kN * 128) + r * 128 + ((cc ^ (r & 7)) << 4)) = w;
    }
    uint4* pz = reinterpret_cast<uint4*>(big + C::kOffP);
    for (int e = tid; e < C::kPBytes / 16; e += 160) pz[e] = make_uint4(0u, 0u, 0u, 0u);
    fence_proxy_async_shared();
    tc::fence_before_sync();
    tc::named_sync(2, 160);
    tc::fence_after_sync();
  }
  const uint32_t tmem = *tmem_base_s;  // valid for every role past named barrier 2

  if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = tc::idesc_bf16(kTile, kN, false, false);
      constexpr uint32_t idO = tc::idesc_bf16(C::kMO, kN, false, true);
      const uint32_t q_s = smem_u32(big + C::kOffQ);
      const uint32_t p_s = smem_u32(big + C::kOffP);
      // S^T(j) = K_j Q^T into S buffer j&1: both operands K-major; 16-wide k
      // steps walk 32 bytes inside a 128-byte swizzle row, then the next block.
      auto issue_s = [&](int j) -> bool {
        const int st = j % C::kStages;
        if (!tc::wait_bounded(&bars[kKVFull0 + st], (j / C::kStages) & 1, abort_flag, p.err, 20)) return false;
        tc::fence_after_sync();
        const uint32_t k_s = smem_u32(big + C::kOffK + st * C::kKVBytes);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint64_t a = tc::sdesc_sw128(k_s + (k >> 2) * kTile * 128 + (k & 3) * 32, 16, 1024);
          const uint64_t b = tc::sdesc_sw128(q_s + (k >> 2) * kN * 128 + (k & 3) * 32, 16, 1024);
          tc::mma_bf16(tmem + C::kTmemS + (j & 1) * kN, a, b, idS, k > 0 ? 1u : 0u);
        }
        tc::mma_commit(&bars[kSFull0 + (j & 1)]);
        return true;
      };
      bool ok = ntiles == 0 || issue_s(0);
      for (int j = 0; ok && j < ntiles; ++j) {
        // Overlap the next tile's S with this tile's softmax (its S buffer was
        // released by the softmax of tile j-1, already waited on below).  With
        // a single K/V stage the next tile only lands after this P V.
        if (C::kStages > 1 && j + 1 < ntiles && !issue_s(j + 1)) break;
        if (!tc::wait_bounded(&bars[kPFull], j & 1, abort_flag, p.err, 21)) break;
        tc::fence_after_sync();
        const int st = j % C::kStages;
        const uint32_t v_s = smem_u32(big + C::kOffV + st * C::kKVBytes);
        // O^T += V^T P^T: A = V^T (MN-major: head dim contiguous; 64-wide
        // blocks kTile*128 bytes apart), B = P^T (K-major over tokens).
#pragma unroll
        for (int k = 0; k < kTile / 16; ++k) {
          const uint64_t b = tc::sdesc_sw128(p_s + (k >> 2) * kN * 128 + (k & 3) * 32, 16, 1024);
#pragma unroll
          for (int mb = 0; mb < D / C::kMO; ++mb) {
            const uint64_t a =
                tc::sdesc_sw128(v_s + mb * (C::kMO / 64) * kTile * 128 + k * 16 * 128, kTile * 128, 1024);
            tc::mma_bf16(tmem + C::kTmemO + mb * kN, a, b, idO, (j > 0 || k > 0) ? 1u : 0u);
          }
        }
        tc::mma_commit(&bars[kODone]);
        tc::mma_commit(&bars[kKVEmpty0 + st]);
        if (C::kStages == 1 && j + 1 < ntiles && !issue_s(j + 1)) break;
      }
    }
  } else if (warp < 4) {
    // ------------------------------------------------------------ softmax
    const int t = threadIdx.x;  // token row of the tile == TMEM lane
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    float m_ref[NREP], l_tok[NREP];
#pragma unroll
    for (int h = 0; h < NREP; ++h) {
      m_ref[h] = -INFINITY;
      l_tok[h] = 0.0f;
    }
    uint8_t* p_s = big + C::kOffP;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      ok = tc::wait_bounded(&bars[kSFull0 + (j & 1)], (j >> 1) & 1, abort_flag, p.err, 30);
      if (!ok) break;
      tc::fence_after_sync();
      float sv[16];
      tmem_ld16(lane_addr + C::kTmemS + (j & 1) * kN, sv);
      const bool valid = j * kTile + t < ntok;
      float* rm = red_max + (j & 1) * 4 * kN;
#pragma unroll
      for (int h = 0; h < NREP; ++h) {
        sv[h] = valid ? sv[h] * p.qscale : -INFINITY;
        const float wm = warp_max(sv[h]);
        if (lane == 0) rm[warp * kN + h] = wm;
      }
      tc::named_sync(1, 128);
      float alpha[NREP];
      bool rescale = false;
#pragma unroll
      for (int h = 0; h < NREP; ++h) {
        const float mt = fmaxf(fmaxf(rm[h], rm[kN + h]), fmaxf(rm[2 * kN + h], rm[3 * kN + h]));
        alpha[h] = 1.0f;
        if (mt > m_ref[h] + kRescaleLog2 || m_ref[h] == -INFINITY) {  // CTA-uniform decision
          alpha[h] = (m_ref[h] == -INFINITY) ? 0.0f : exp2f(m_ref[h] - mt);
          m_ref[h] = mt;  // finite: every tile holds a valid token
          rescale |= j > 0;
        }
        sv[h] = exp2f(sv[h] - m_ref[h]);  // masked tokens: exp2(-inf) = 0
        l_tok[h] = l_tok[h] * alpha[h] + sv[h];
      }
      if (j > 0) {
        // The P^T buffer (and O^T, when rescaling) is busy until the
        // previous P V finishes.
        ok = tc::wait_bounded(&bars[kODone], (j - 1) & 1, abort_flag, p.err, 31);
        if (!ok) break;
        tc::fence_after_sync();
        if (rescale) {
#pragma unroll
          for (int mb = 0; mb < D / C::kMO; ++mb) {
            float ov[16];
            tmem_ld16(lane_addr + C::kTmemO + mb * kN, ov);
#pragma unroll
            for (int h = 0; h < NREP; ++h) ov[h] *= alpha[h];
            tmem_st16(lane_addr + C::kTmemO + mb * kN, ov);
          }
          tc::tmem_st_wait();
        }
      }
      // P^T[h][t] (bf16) in the K-major swizzled layout: 64-token sub-tiles
      // of 16 rows x 128 bytes; 16-byte chunk index XOR (row % 8).
      {
        const int sub = t >> 6, col = t & 63;
#pragma unroll
        for (int h = 0; h < NREP; ++h) {
          const int off = sub * (kN * 128) + h * 128 + ((((col >> 3) ^ (h & 7))) << 4) + (col & 7) * 2;
          *reinterpret_cast<__nv_bfloat16*>(p_s + off) = __float2bfloat16_rn(sv[h]);
        }
      }
      fence_proxy_async_shared();
      tc::fence_before_sync();
      tc::mbar_arrive(&bars[kPFull]);
    }

    // ---- epilogue: l per head over the CTA; O^T rows of this thread's lane.
    if (ok && ntiles > 0) ok = tc::wait_bounded(&bars[kODone], (ntiles - 1) & 1, abort_flag, p.err, 32);
    tc::fence_after_sync();
    const bool have_o = __all_sync(0xffffffffu, ok) && ntiles > 0;  // warp-uniform for tcgen05.ld
#pragma unroll
    for (int h = 0; h < NREP; ++h) {
      const float ws = warp_sum(l_tok[h]);
      if (lane == 0) red_sum[warp * kN + h] = ws;
    }
    tc::named_sync(1, 128);
    float l_cta[NREP];
#pragma unroll
    for (int h = 0; h < NREP; ++h)
      l_cta[h] = red_sum[h] + red_sum[kN + h] + red_sum[2 * kN + h] + red_sum[3 * kN + h];

    const int64_t head0 = static_cast<int64_t>(s) * p.hq + g * NREP;
    // Rows of O^T this thread holds: M=64 puts row d in lane (d % 16) + 32 (d / 16);
    // M=128 puts row d in lane d; D = 256 uses two M=128 blocks 16 columns apart.
    const bool holds = (C::kMO == 64) ? (lane < 16) : true;
    const int d_base = (C::kMO == 64) ? warp * 16 + lane : warp * 32 + lane;
#pragma unroll
    for (int mb = 0; mb < D / C::kMO; ++mb) {
      float ov[16];
      if (have_o) {
        tmem_ld16(lane_addr + C::kTmemO + mb * kN, ov);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) ov[i] = 0.0f;
      }
      const int d = d_base + mb * 128;
      if (!holds) continue;
#pragma unroll
      for (int h = 0; h < NREP; ++h) {
        if (n_splits == 1) {
          const float r = finalize(ov[h], l_cta[h], m_ref[h], p.phantom);
          if (p.o_f32) static_cast<float*>(p.o)[(head0 + h) * D + d] = r;
          else static_cast<__nv_bfloat16*>(p.o)[(head0 + h) * D + d] = __float2bfloat16_rn(r);
        } else {
          const int64_t slot = (head0 + h) * p.max_splits + split;
          p.ws_o[slot * D + d] = ov[h];
          if (d == 0) {
            p.ws_ml[slot * 2 + 0] = m_ref[h];
            p.ws_ml[slot * 2 + 1] = l_cta[h];
          }
        }
      }
    }

    if (n_splits > 1) {
      // ---- split combine: the last CTA of (sequence, kv head) merges in split order.
      __threadfence();
      tc::named_sync(1, 128);
      if (t == 0) {
        const unsigned int ticket = atomicAdd(&p.ws_cnt[s * p.hkv + g], 1u);
        *last_flag = (ticket == static_cast<unsigned int>(n_splits - 1)) ? 1 : 0;
      }
      tc::named_sync(1, 128);
      if (*last_flag) {
        __threadfence();
        for (int e = t; e < NREP * D; e += 128) {
          const int h = e / D, d = e - (e / D) * D;
          const int64_t slot0 = (head0 + h) * p.max_splits;
          float mall = -INFINITY;
          for (int jj = 0; jj < n_splits; ++jj) mall = fmaxf(mall, ld_cg(p.ws_ml + (slot0 + jj) * 2));
          float o = 0.0f, l = 0.0f;
          if (mall != -INFINITY) {
            for (int jj = 0; jj < n_splits; ++jj) {
              const float mj = ld_cg(p.ws_ml + (slot0 + jj) * 2);
              if (mj == -INFINITY) continue;
              const float a = exp2f(mj - mall);
              o += ld_cg(p.ws_o + (slot0 + jj) * D + d) * a;
              l += ld_cg(p.ws_ml + (slot0 + jj) * 2 + 1) * a;
            }
          }
          const float r = finalize(o, l, mall, p.phantom);
          if (p.o_f32) static_cast<float*>(p.o)[(head0 + h) * D + d] = r;
          else static_cast<__nv_bfloat16*>(p.o)[(head0 + h) * D + d] = __float2bfloat16_rn(r);
        }
        if (t == 0) p.ws_cnt[s * p.hkv + g] = 0u;  // ready for the next launch on this workspace
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

template <int D, int NREP>
int launch_decode(const CUtensorMap& tkv, const DecodeParams& prm, int n_seqs, cudaStream_t stream) {
  using C = DCfg<D>;
  auto kern = paged_decode_kernel<D, NREP>;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    MTN_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem),
                 "cudaFuncSetAttribute(decode)");
    configured[dev] = true;
  }
  dim3 grid(prm.max_splits, prm.hkv, n_seqs);
  kern<<<grid, kThreads, C::kSmem, stream>>>(tkv, prm);
  return check_launch("paged_decode_kernel");
}

template <int D>
int dispatch_nrep(int nrep, const CUtensorMap& tkv, const DecodeParams& prm, int n_seqs, cudaStream_t stream) {
  switch (nrep) {
    case 1: return launch_decode<D, 1>(tkv, prm, n_seqs, stream);
    case 2: return launch_decode<D, 2>(tkv, prm, n_seqs, stream);
    case 3: return launch_decode<D, 3>(tkv, prm, n_seqs, stream);
    case 4: return launch_decode<D, 4>(tkv, prm, n_seqs, stream);
    case 5: return launch_decode<D, 5>(tkv, prm, n_seqs, stream);
    case 6: return launch_decode<D, 6>(tkv, prm, n_seqs, stream);
    case 7: return launch_decode<D, 7>(tkv, prm, n_seqs, stream);
    case 8: return launch_decode<D, 8>(tkv, prm, n_seqs, stream);
    default: return set_error(MTN_EINVAL, "paged decode: query heads per kv head %d not in [1,8]", nrep);
  }
}

int effective_split(int page_size, int pages_per_split) {
  const int tp = kTile / page_size;
  if (pages_per_split <= 0) pages_per_split = tp;
  pages_per_split = std::min(pages_per_split, DCfg<64>::kMaxSplitPages);
  return ((pages_per_split + tp - 1) / tp) * tp;
}

}  // namespace
}  // namespace mtn

using mtn::set_error;

extern "C" {

size_t mtn_paged_decode_workspace_bytes(int32_t n_seqs, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                        int32_t max_pages_per_seq, int32_t pages_per_split) {
  if (n_seqs <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || max_pages_per_seq < 0) return 0;
  // Splits are rounded up to whole 128-token tiles, which only lowers the
  // split count, so sizing with the pages_per_split given (at least 1) is safe.
  const int64_t pps = pages_per_split > 0 ? pages_per_split : 1;
  const int64_t max_splits = std::max<int64_t>(1, (max_pages_per_seq + pps - 1) / pps);
  const int64_t slots = static_cast<int64_t>(n_seqs) * num_q_heads * max_splits;
  size_t bytes = static_cast<size_t>(slots) * head_dim * 4;   // ws_o
  bytes += static_cast<size_t>(slots) * 2 * 4;                  // ws_ml
  bytes += static_cast<size_t>(n_seqs) * num_kv_heads * 4;      // arrival counters
  return (bytes + 255) & ~static_cast<size_t>(255);
}

int32_t mtn_paged_decode_default_split(const mtn_kv_layout* pool, int32_t n_seqs, int64_t total_pages,
                                       int32_t max_pages_per_seq, int32_t num_q_heads) {
  (void)num_q_heads;
  if (pool == nullptr || pool->page_size <= 0 || n_seqs <= 0 || mtn::kTile % pool->page_size != 0) return 0;
  const int tp = mtn::kTile / pool->page_size;
  // About six CTAs per SM of (page, kv head) work: enough to cover the
  // device twice with the ~3 resident CTAs per SM, few partials to merge.
  const int64_t target = static_cast<int64_t>(mtn::sm_count()) * 6;
  const int64_t units = std::max<int64_t>(1, total_pages) * pool->num_kv_heads;
  int64_t pps = (units + target - 1) / target;
  pps = std::max<int64_t>(pps, tp);
  pps = std::min<int64_t>(pps, std::max(max_pages_per_seq, 1));
  return mtn::effective_split(pool->page_size, static_cast<int>(pps));
}

int mtn_paged_decode(const mtn_kv_layout* pool, int32_t layer, const void* q, int32_t q_dtype, void* o,
                     int32_t o_dtype, int32_t n_seqs, int32_t num_q_heads, const int32_t* kv_indptr,
                     const int32_t* kv_indices, const int32_t* seq_lens, int32_t max_pages_per_seq,
                     int32_t pages_per_split, float scale, uint32_t flags, void* workspace, size_t workspace_bytes,
                     void* stream) {
  int st = mtn::validate_layout(pool, layer, "mtn_paged_decode");
  if (st != MTN_OK) return st;
  MTN_CHECK_ARG(n_seqs >= 0 && n_seqs <= 65535, "mtn_paged_decode: n_seqs %d outside [0, 65535]", n_seqs);
  if (n_seqs == 0) return MTN_OK;
  MTN_CHECK_ARG(q && o && kv_indptr && kv_indices && seq_lens, "mtn_paged_decode: null pointer");
  MTN_CHECK_ARG(q_dtype == MTN_DTYPE_BF16 || q_dtype == MTN_DTYPE_F32, "mtn_paged_decode: bad q dtype");
  MTN_CHECK_ARG(o_dtype == MTN_DTYPE_BF16 || o_dtype == MTN_DTYPE_F32, "mtn_paged_decode: bad o dtype");
  MTN_CHECK_ARG(num_q_heads > 0 && num_q_heads % pool->num_kv_heads == 0,
                "mtn_paged_decode: %d query heads not a multiple of %d kv heads", num_q_heads, pool->num_kv_heads);
  MTN_CHECK_ARG(pool->num_kv_heads <= 65535, "mtn_paged_decode: too many kv heads");
  const int D = pool->head_dim;
  MTN_CHECK_ARG(pool->page_size % 8 == 0 && mtn::kTile % pool->page_size == 0,
                "mtn_paged_decode: page_size %d must be a multiple of 8 dividing %d", pool->page_size, mtn::kTile);
  MTN_CHECK_ARG(max_pages_per_seq >= 0, "mtn_paged_decode: max_pages_per_seq < 0");
  MTN_CHECK_ARG((reinterpret_cast<uintptr_t>(q) & 15) == 0 && (reinterpret_cast<uintptr_t>(o) & 15) == 0,
                "mtn_paged_decode: q/o must be 16-byte aligned");
  const int pps = mtn::effective_split(pool->page_size, pages_per_split);
  const int max_splits = std::max(1, (max_pages_per_seq + pps - 1) / pps);
  MTN_CHECK_ARG(max_splits <= (1 << 20), "mtn_paged_decode: too many splits");
  const size_t need = mtn_paged_decode_workspace_bytes(n_seqs, num_q_heads, pool->num_kv_heads, D,
                                                       max_pages_per_seq, pps);
  if (max_splits > 1) {
    MTN_CHECK_ARG(workspace != nullptr && workspace_bytes >= need,
                  "mtn_paged_decode: workspace of %zu bytes < %zu needed", workspace_bytes, need);
    MTN_CHECK_ARG((reinterpret_cast<uintptr_t>(workspace) & 15) == 0, "mtn_paged_decode: workspace alignment");
  }
  CUtensorMap tkv;
  st = mtn::pool_tensor_map(pool, &tkv);
  if (st != MTN_OK) return st;

  mtn::DecodeParams prm{};
  const int64_t rows_per_block = pool->num_pages * pool->num_kv_heads * pool->page_size;
  prm.row_k = (static_cast<int64_t>(layer) * 2 + 0) * rows_per_block;
  prm.row_v = (static_cast<int64_t>(layer) * 2 + 1) * rows_per_block;
  prm.num_pages = pool->num_pages;
  prm.hkv = pool->num_kv_heads;
  prm.ps = pool->page_size;
  prm.hq = num_q_heads;
  prm.q = q;
  prm.o = o;
  prm.q_f32 = q_dtype == MTN_DTYPE_F32;
  prm.o_f32 = o_dtype == MTN_DTYPE_F32;
  prm.kv_indptr = kv_indptr;
  prm.kv_indices = kv_indices;
  prm.seq_lens = seq_lens;
  prm.pages_per_split = pps;
  prm.max_splits = max_splits;
  prm.qscale = scale * mtn::kLog2e;
  prm.phantom = (flags & MTN_ATTN_PHANTOM_ZERO_SLOT) ? 1 : 0;
  if (max_splits > 1) {
    const int64_t slots = static_cast<int64_t>(n_seqs) * num_q_heads * max_splits;
    prm.ws_o = static_cast<float*>(workspace);
    prm.ws_ml = prm.ws_o + slots * D;
    prm.ws_cnt = reinterpret_cast<unsigned int*>(prm.ws_ml + slots * 2);
  }
  prm.err = mtn::device_error_ptr();
  const int nrep = num_q_heads / pool->num_kv_heads;
  auto s = static_cast<cudaStream_t>(stream);
  switch (D) {
    case 64: return mtn::dispatch_nrep<64>(nrep, tkv, prm, n_seqs, s);
    case 128: return mtn::dispatch_nrep<128>(nrep, tkv, prm, n_seqs, s);
    default: return mtn::dispatch_nrep<256>(nrep, tkv, prm, n_seqs, s);
  }
}

}  // extern "C"
