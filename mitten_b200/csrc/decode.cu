// Paged GQA/MQA decode attention for sm_100a (one query token per sequence).
//
// Replaces the decode-step attention of qwen model.rs:394-416: GQA head
// mapping h -> h / n_rep (model.rs:398-408), scores q.k * scale
// (model.rs:298, 413), softmax over every key including the reference's
// all-zero first row (model.rs:207-220, flag MTN_ATTN_PHANTOM_ZERO_SLOT),
// output P.V (model.rs:416).  No causal mask is needed for one query token:
// generate_causal_mask (model.rs:542-555) masks nothing on the last row.
//
// Design (HBM-bound, CUDA cores):
//   - grid = (split, kv head, sequence).  A CTA owns `pages_per_split`
//     consecutive pages of one sequence for one KV head and all n_rep query
//     heads that share it, so every K/V byte is read from HBM once.
//   - Pages are staged into shared memory by the TMA engine with 1-D bulk
//     copies (cp.async.bulk, one per page per K/V: the pool keeps each
//     (page, kv head) slab contiguous), STAGES tiles in flight, completion
//     tracked by mbarrier transaction counts.
//   - QK: lane = token; the lane walks the head dim in 16-byte chunks
//     starting at chunk (lane mod chunks) so the 8 lanes of a shared-memory
//     phase hit 8 different bank groups; Q (pre-scaled by scale*log2 e) is
//     read as a broadcast; packed f32x2 FMAs (FFMA2).
//   - Online softmax per warp in the exp2 domain (warp-shuffle max), P is
//     written once per tile to shared memory.
//   - PV: lane = (16-byte dim chunk, token group); FFMA2 over bf16 V rows.
//   - Fixed-order combine: warps of a CTA merge in warp order; splits of a
//     sequence write (m, l, O) partials to the workspace and the last CTA
//     to arrive (atomic ticket, no spinning) merges them in split order, so
//     the result does not depend on CTA scheduling.
#include <cfloat>

#include "common.cuh"

namespace mtn {
namespace {

constexpr float kLog2e = 1.4426950408889634f;

struct DecodeParams {
  const __nv_bfloat16* kpool;  // K block of the layer: [num_pages][hkv][ps][D]
  const __nv_bfloat16* vpool;  // V block of the layer
  int64_t num_pages;
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
  float* ws_o;         // [n_seqs][hq][max_splits][D]
  float* ws_ml;        // [n_seqs][hq][max_splits][2]
  unsigned int* ws_cnt;  // [n_seqs][hkv]
  int* err;
};

template <int D, int NREP, int NWARPS, int TILE_TOK, int STAGES>
struct DecodeCfg {
  static constexpr int kThreads = NWARPS * 32;
  static constexpr int kChunks = D / 8;             // 16-byte chunks per row
  static constexpr int kTokPerWarp = TILE_TOK / NWARPS;
  static constexpr int kTT = kTokPerWarp / 32;       // tokens per lane in QK
  static constexpr int kTG = 32 / kChunks > 0 ? 32 / kChunks : 1;  // token groups in PV
  static constexpr int kNrep2 = (NREP + 1) & ~1;
  static constexpr int kStageBytes = TILE_TOK * D * 2;  // one of K or V
  static constexpr int kOffQ = STAGES * 2 * kStageBytes;
  static constexpr int kOffP = kOffQ + NREP * D * 4;
  static constexpr int kOffBar = (kOffP + NWARPS * kTokPerWarp * kNrep2 * 8 + 15) & ~15;
  static constexpr int kOffFlag = kOffBar + STAGES * 8;
  static constexpr int kSmem = kOffFlag + 16;
  // Cross-warp combine buffers alias the stage area after the main loop.
  static constexpr int kCombBytes = NWARPS * NREP * (D + 2) * 4;
  static_assert(kCombBytes <= STAGES * 2 * kStageBytes, "combine buffer must fit in the stage area");
  static_assert(kTokPerWarp % 32 == 0, "tile must give each lane whole tokens");
  static_assert(D % 64 == 0, "head_dim must be a multiple of 64");
};

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

template <int D, int NREP, int NWARPS, int TILE_TOK, int STAGES>
__global__ void __launch_bounds__(NWARPS * 32)
    paged_decode_kernel(const __grid_constant__ DecodeParams p) {
  using C = DecodeCfg<D, NREP, NWARPS, TILE_TOK, STAGES>;
  extern __shared__ __align__(128) uint8_t smem[];
  float4* q_s = reinterpret_cast<float4*>(smem + C::kOffQ);  // [NREP][2][kChunks]
  float2* p_s = reinterpret_cast<float2*>(smem + C::kOffP);  // [NWARPS][kTokPerWarp][kNrep2]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  int* flag = reinterpret_cast<int*>(smem + C::kOffFlag);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split = blockIdx.x;
  const int g = blockIdx.y;
  const int s = blockIdx.z;

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
  const int tok_end = min(seq_len, pg1 * p.ps);
  const int ntok = max(0, tok_end - tok_begin);
  const int ntiles = (ntok + TILE_TOK - 1) / TILE_TOK;
  const int tile_pages = TILE_TOK / p.ps;
  const int page_elems = p.ps * D;
  const uint32_t page_bytes = static_cast<uint32_t>(page_elems) * 2u;

  // Producer: warp 0 stages tile `i` (all its pages, K and V) into stage i % STAGES.
  auto issue_tile = [&](int i) {
    const int st = i % STAGES;
    const int tp0 = pg0 + i * tile_pages;
    const int tp1 = min(pg1, tp0 + tile_pages);
    if (lane == 0) mbar_arrive_expect_tx(&bars[st], static_cast<uint32_t>(tp1 - tp0) * page_bytes * 2u);
    __syncwarp();
    __nv_bfloat16* kst = reinterpret_cast<__nv_bfloat16*>(smem + st * 2 * C::kStageBytes);
    __nv_bfloat16* vst = kst + TILE_TOK * D;
    for (int j = tp0 + lane; j < tp1; j += 32) {
      int64_t page = p.kv_indices[pbeg + j];
      if (page < 0 || page >= p.num_pages) {
        record_error(p.err, kDevErrBadPage, s);
        page = 0;
      }
      const int64_t off = (page * p.hkv + g) * page_elems;
      bulk_g2s(kst + (j - tp0) * page_elems, p.kpool + off, page_bytes, &bars[st]);
      bulk_g2s(vst + (j - tp0) * page_elems, p.vpool + off, page_bytes, &bars[st]);
    }
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) mbar_init(&bars[i], 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (warp == 0) {
    for (int i = 0; i < min(STAGES, ntiles); ++i) issue_tile(i);
  }

  // Q for the n_rep heads of this KV head, pre-scaled, as f32 [h][half][chunk].
  for (int e = threadIdx.x; e < NREP * C::kChunks * 2; e += C::kThreads) {
    const int h = e / (C::kChunks * 2);
    const int rem = e - h * C::kChunks * 2;
    const int c = rem >> 1, half = rem & 1;
    const int64_t qoff = (static_cast<int64_t>(s) * p.hq + g * NREP + h) * D + c * 8 + half * 4;
    float4 v;
    if (p.q_f32) {
      v = *reinterpret_cast<const float4*>(static_cast<const float*>(p.q) + qoff);
    } else {
      const uint2 w = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(p.q) + qoff);
      const float2 a = bf2_to_f2(w.x), b = bf2_to_f2(w.y);
      v = make_float4(a.x, a.y, b.x, b.y);
    }
    v.x *= p.qscale; v.y *= p.qscale; v.z *= p.qscale; v.w *= p.qscale;
    q_s[(h * 2 + half) * C::kChunks + c] = v;
  }
  __syncthreads();

  // Per-warp online-softmax state (m is warp-uniform).
  float m_run[NREP], l_run[NREP];
  float2 oacc[NREP][4];
#pragma unroll
  for (int h = 0; h < NREP; ++h) {
    m_run[h] = -INFINITY;
    l_run[h] = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) oacc[h][k] = make_float2(0.0f, 0.0f);
  }
  const int dc = lane % C::kChunks;  // PV: this lane's 16-byte dim chunk
  const int tg = lane / C::kChunks;  // PV: this lane's token group
  float2* pw = p_s + warp * C::kTokPerWarp * C::kNrep2;

  for (int i = 0; i < ntiles; ++i) {
    const int st = i % STAGES;
    mbar_wait_bounded(&bars[st], static_cast<uint32_t>((i / STAGES) & 1), p.err, 1);
    const uint4* kt = reinterpret_cast<const uint4*>(smem + st * 2 * C::kStageBytes);
    const uint4* vt = reinterpret_cast<const uint4*>(smem + st * 2 * C::kStageBytes + C::kStageBytes);
    const int nvalid = min(TILE_TOK, ntok - i * TILE_TOK);
    const int wt0 = warp * C::kTokPerWarp;

    // ---- S = Q K^T for this lane's tokens.
    float2 acc[C::kTT][NREP];
#pragma unroll
    for (int j = 0; j < C::kTT; ++j)
#pragma unroll
      for (int h = 0; h < NREP; ++h) acc[j][h] = make_float2(0.0f, 0.0f);

#pragma unroll 4
    for (int c = 0; c < C::kChunks; ++c) {
      const int cc = (c + lane) & (C::kChunks - 1);
      float2 kf[C::kTT][4];
#pragma unroll
      for (int j = 0; j < C::kTT; ++j) {
        const uint4 kw = kt[(wt0 + lane + 32 * j) * C::kChunks + cc];
        kf[j][0] = bf2_to_f2(kw.x);
        kf[j][1] = bf2_to_f2(kw.y);
        kf[j][2] = bf2_to_f2(kw.z);
        kf[j][3] = bf2_to_f2(kw.w);
      }
#pragma unroll
      for (int h = 0; h < NREP; ++h) {
        const float4 qa = q_s[(h * 2 + 0) * C::kChunks + cc];
        const float4 qb = q_s[(h * 2 + 1) * C::kChunks + cc];
#pragma unroll
        for (int j = 0; j < C::kTT; ++j) {
          acc[j][h] = ffma2(make_float2(qa.x, qa.y), kf[j][0], acc[j][h]);
          acc[j][h] = ffma2(make_float2(qa.z, qa.w), kf[j][1], acc[j][h]);
          acc[j][h] = ffma2(make_float2(qb.x, qb.y), kf[j][2], acc[j][h]);
          acc[j][h] = ffma2(make_float2(qb.z, qb.w), kf[j][3], acc[j][h]);
        }
      }
    }

    // ---- online softmax (exp2 domain; scores already carry scale*log2 e).
    float alpha[NREP];
#pragma unroll
    for (int h = 0; h < NREP; ++h) {
      float sc[C::kTT];
      float mt = -INFINITY;
#pragma unroll
      for (int j = 0; j < C::kTT; ++j) {
        const bool valid = (wt0 + lane + 32 * j) < nvalid;
        sc[j] = valid ? acc[j][h].x + acc[j][h].y : -INFINITY;
        mt = fmaxf(mt, sc[j]);
      }
      mt = warp_max(mt);
      const float mn = fmaxf(m_run[h], mt);
      float psum = 0.0f;
      if (mn == -INFINITY) {
        alpha[h] = 1.0f;
#pragma unroll
        for (int j = 0; j < C::kTT; ++j) pw[(lane + 32 * j) * C::kNrep2 + h] = make_float2(0.0f, 0.0f);
      } else {
        alpha[h] = exp2f(m_run[h] - mn);
#pragma unroll
        for (int j = 0; j < C::kTT; ++j) {
          const float pv = exp2f(sc[j] - mn);
          psum += pv;
          pw[(lane + 32 * j) * C::kNrep2 + h] = make_float2(pv, pv);
        }
      }
      l_run[h] = l_run[h] * alpha[h] + psum;
      m_run[h] = mn;
    }
    __syncwarp();

    // ---- O = alpha * O + P V over this warp's tokens.
#pragma unroll
    for (int h = 0; h < NREP; ++h) {
      const float2 a2 = make_float2(alpha[h], alpha[h]);
#pragma unroll
      for (int k = 0; k < 4; ++k) oacc[h][k] = __fmul2_rn(oacc[h][k], a2);
    }
    const int nw = min(C::kTokPerWarp, max(0, nvalid - wt0));
#pragma unroll 4
    for (int t = tg; t < nw; t += C::kTG) {
      const uint4 vw = vt[(wt0 + t) * C::kChunks + dc];
      const float2 v0 = bf2_to_f2(vw.x), v1 = bf2_to_f2(vw.y), v2 = bf2_to_f2(vw.z), v3 = bf2_to_f2(vw.w);
      const float4* pt = reinterpret_cast<const float4*>(pw + t * C::kNrep2);
#pragma unroll
      for (int h2 = 0; h2 < C::kNrep2 / 2; ++h2) {
        const float4 pp = pt[h2];
        const float2 pa = make_float2(pp.x, pp.y);
        const float2 pb = make_float2(pp.z, pp.w);
        const int ha = 2 * h2, hb = 2 * h2 + 1;
        oacc[ha][0] = ffma2(pa, v0, oacc[ha][0]);
        oacc[ha][1] = ffma2(pa, v1, oacc[ha][1]);
        oacc[ha][2] = ffma2(pa, v2, oacc[ha][2]);
        oacc[ha][3] = ffma2(pa, v3, oacc[ha][3]);
        if (hb < NREP) {
          oacc[hb][0] = ffma2(pb, v0, oacc[hb][0]);
          oacc[hb][1] = ffma2(pb, v1, oacc[hb][1]);
          oacc[hb][2] = ffma2(pb, v2, oacc[hb][2]);
          oacc[hb][3] = ffma2(pb, v3, oacc[hb][3]);
        }
      }
    }
    __syncthreads();  // every warp is done with stage `st` and with its P slots
    if (warp == 0 && i + STAGES < ntiles) issue_tile(i + STAGES);
  }

  // ---- reduce the PV token groups inside the warp, and l across lanes.
#pragma unroll
  for (int o = C::kChunks; o < 32; o <<= 1) {
#pragma unroll
    for (int h = 0; h < NREP; ++h)
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        oacc[h][k].x += __shfl_xor_sync(0xffffffffu, oacc[h][k].x, o);
        oacc[h][k].y += __shfl_xor_sync(0xffffffffu, oacc[h][k].y, o);
      }
  }
#pragma unroll
  for (int h = 0; h < NREP; ++h) l_run[h] = warp_sum(l_run[h]);

  // ---- cross-warp combine, in warp order (buffers alias the stage area).
  float* comb_o = reinterpret_cast<float*>(smem);          // [NWARPS][NREP][D]
  float* comb_ml = comb_o + NWARPS * NREP * D;              // [NWARPS][NREP][2]
  if (tg == 0) {
#pragma unroll
    for (int h = 0; h < NREP; ++h) {
      float4* dst = reinterpret_cast<float4*>(comb_o + (warp * NREP + h) * D + dc * 8);
      dst[0] = make_float4(oacc[h][0].x, oacc[h][0].y, oacc[h][1].x, oacc[h][1].y);
      dst[1] = make_float4(oacc[h][2].x, oacc[h][2].y, oacc[h][3].x, oacc[h][3].y);
    }
  }
  if (lane == 0) {
#pragma unroll
    for (int h = 0; h < NREP; ++h) {
      comb_ml[(warp * NREP + h) * 2 + 0] = m_run[h];
      comb_ml[(warp * NREP + h) * 2 + 1] = l_run[h];
    }
  }
  __syncthreads();

  const int64_t head0 = static_cast<int64_t>(s) * p.hq + g * NREP;  // first q head of this CTA
  for (int e = threadIdx.x; e < NREP * D; e += C::kThreads) {
    const int h = e / D, d = e - (e / D) * D;
    float mc = -INFINITY;
#pragma unroll
    for (int w = 0; w < NWARPS; ++w) mc = fmaxf(mc, comb_ml[(w * NREP + h) * 2]);
    float o = 0.0f, l = 0.0f;
    if (mc != -INFINITY) {
#pragma unroll
      for (int w = 0; w < NWARPS; ++w) {
        const float mw = comb_ml[(w * NREP + h) * 2];
        if (mw == -INFINITY) continue;
        const float a = exp2f(mw - mc);
        o += comb_o[(w * NREP + h) * D + d] * a;
        l += comb_ml[(w * NREP + h) * 2 + 1] * a;
      }
    }
    if (n_splits == 1) {
      const float r = finalize(o, l, mc, p.phantom);
      if (p.o_f32) static_cast<float*>(p.o)[(head0 + h) * D + d] = r;
      else static_cast<__nv_bfloat16*>(p.o)[(head0 + h) * D + d] = __float2bfloat16_rn(r);
    } else {
      const int64_t slot = (head0 + h) * p.max_splits + split;
      p.ws_o[slot * D + d] = o;
      if (d == 0) {
        p.ws_ml[slot * 2 + 0] = mc;
        p.ws_ml[slot * 2 + 1] = l;
      }
    }
  }
  if (n_splits == 1) return;

  // ---- split combine: the last CTA of (sequence, kv head) merges in split order.
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int ticket = atomicAdd(&p.ws_cnt[s * p.hkv + g], 1u);
    *flag = (ticket == static_cast<unsigned int>(n_splits - 1)) ? 1 : 0;
  }
  __syncthreads();
  if (*flag == 0) return;
  __threadfence();
  for (int e = threadIdx.x; e < NREP * D; e += C::kThreads) {
    const int h = e / D, d = e - (e / D) * D;
    const int64_t slot0 = (head0 + h) * p.max_splits;
    float mall = -INFINITY;
    for (int j = 0; j < n_splits; ++j) mall = fmaxf(mall, ld_cg(p.ws_ml + (slot0 + j) * 2));
    float o = 0.0f, l = 0.0f;
    if (mall != -INFINITY) {
      for (int j = 0; j < n_splits; ++j) {
        const float mj = ld_cg(p.ws_ml + (slot0 + j) * 2);
        if (mj == -INFINITY) continue;
        const float a = exp2f(mj - mall);
        o += ld_cg(p.ws_o + (slot0 + j) * D + d) * a;
        l += ld_cg(p.ws_ml + (slot0 + j) * 2 + 1) * a;
      }
    }
    const float r = finalize(o, l, mall, p.phantom);
    if (p.o_f32) static_cast<float*>(p.o)[(head0 + h) * D + d] = r;
    else static_cast<__nv_bfloat16*>(p.o)[(head0 + h) * D + d] = __float2bfloat16_rn(r);
  }
  if (threadIdx.x == 0) p.ws_cnt[s * p.hkv + g] = 0u;  // ready for the next launch on this workspace
}

// Per-head-dim launch shapes: 64 KiB of K/V stages per CTA.
template <int D> struct Shape;
template <> struct Shape<64> { static constexpr int kWarps = 4, kTile = 128, kStages = 2; };
template <> struct Shape<128> { static constexpr int kWarps = 2, kTile = 64, kStages = 2; };
template <> struct Shape<256> { static constexpr int kWarps = 1, kTile = 32, kStages = 2; };

template <int D, int NREP>
int launch_decode(const DecodeParams& prm, int n_seqs, cudaStream_t stream) {
  using S = Shape<D>;
  using C = DecodeCfg<D, NREP, S::kWarps, S::kTile, S::kStages>;
  auto kern = paged_decode_kernel<D, NREP, S::kWarps, S::kTile, S::kStages>;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    MTN_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem),
                 "cudaFuncSetAttribute(decode)");
    configured[dev] = true;
  }
  dim3 grid(prm.max_splits, prm.hkv, n_seqs);
  kern<<<grid, C::kThreads, C::kSmem, stream>>>(prm);
  return check_launch("paged_decode_kernel");
}

template <int D>
int dispatch_nrep(int nrep, const DecodeParams& prm, int n_seqs, cudaStream_t stream) {
  switch (nrep) {
    case 1: return launch_decode<D, 1>(prm, n_seqs, stream);
    case 2: return launch_decode<D, 2>(prm, n_seqs, stream);
    case 3: return launch_decode<D, 3>(prm, n_seqs, stream);
    case 4: return launch_decode<D, 4>(prm, n_seqs, stream);
    case 5: return launch_decode<D, 5>(prm, n_seqs, stream);
    case 6: return launch_decode<D, 6>(prm, n_seqs, stream);
    case 7: return launch_decode<D, 7>(prm, n_seqs, stream);
    case 8: return launch_decode<D, 8>(prm, n_seqs, stream);
    default: return set_error(MTN_EINVAL, "paged decode: query heads per kv head %d not in [1,8]", nrep);
  }
}

int tile_pages_for(int head_dim, int page_size) {
  const int tile = head_dim == 64 ? Shape<64>::kTile : head_dim == 128 ? Shape<128>::kTile : Shape<256>::kTile;
  return tile / page_size;
}

int tile_tokens_for(int head_dim) {
  return head_dim == 64 ? Shape<64>::kTile : head_dim == 128 ? Shape<128>::kTile : Shape<256>::kTile;
}

int effective_split(int head_dim, int page_size, int pages_per_split) {
  const int tp = tile_pages_for(head_dim, page_size);
  if (pages_per_split <= 0) pages_per_split = tp;
  return ((pages_per_split + tp - 1) / tp) * tp;
}

}  // namespace
}  // namespace mtn

using mtn::set_error;

extern "C" {

size_t mtn_paged_decode_workspace_bytes(int32_t n_seqs, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                        int32_t max_pages_per_seq, int32_t pages_per_split) {
  if (n_seqs <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || max_pages_per_seq < 0) return 0;
  // Page size only changes the rounding of pages_per_split; size for the
  // smallest legal tile (page_size 16 for every head dim) conservatively
  // by using pages_per_split as given, at least 1.
  const int64_t pps = pages_per_split > 0 ? pages_per_split : 1;
  const int64_t max_splits = std::max<int64_t>(1, (max_pages_per_seq + pps - 1) / pps);
  const int64_t slots = static_cast<int64_t>(n_seqs) * num_q_heads * max_splits;
  size_t bytes = static_cast<size_t>(slots) * head_dim * 4;               // ws_o
  bytes += static_cast<size_t>(slots) * 2 * 4;                              // ws_ml
  bytes += static_cast<size_t>(n_seqs) * num_kv_heads * 4;                  // counters
  return (bytes + 255) & ~static_cast<size_t>(255);
}

int32_t mtn_paged_decode_default_split(const mtn_kv_layout* pool, int32_t n_seqs, int64_t total_pages,
                                       int32_t max_pages_per_seq, int32_t num_q_heads) {
  (void)num_q_heads;
  if (pool == nullptr || pool->page_size <= 0 || n_seqs <= 0) return 0;
  if (pool->head_dim != 64 && pool->head_dim != 128 && pool->head_dim != 256) return 0;
  if (mtn::tile_tokens_for(pool->head_dim) % pool->page_size != 0) return 0;
  const int tp = mtn::tile_pages_for(pool->head_dim, pool->page_size);
  // Aim for about four resident CTA slots' worth of work items per SM.
  const int64_t target = static_cast<int64_t>(mtn::sm_count()) * 8;
  const int64_t units = std::max<int64_t>(1, total_pages) * pool->num_kv_heads;
  int64_t pps = (units + target - 1) / target;
  pps = std::max<int64_t>(pps, tp);
  pps = std::min<int64_t>(pps, std::max(max_pages_per_seq, 1));
  return mtn::effective_split(pool->head_dim, pool->page_size, static_cast<int>(pps));
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
  const int D = pool->head_dim;
  MTN_CHECK_ARG(mtn::tile_tokens_for(D) % pool->page_size == 0,
                "mtn_paged_decode: page_size %d must divide the %d-token tile", pool->page_size,
                mtn::tile_tokens_for(D));
  MTN_CHECK_ARG(max_pages_per_seq >= 0, "mtn_paged_decode: max_pages_per_seq < 0");
  MTN_CHECK_ARG((reinterpret_cast<uintptr_t>(q) & 15) == 0 && (reinterpret_cast<uintptr_t>(o) & 15) == 0,
                "mtn_paged_decode: q/o must be 16-byte aligned");
  const int pps = mtn::effective_split(D, pool->page_size, pages_per_split);
  const int max_splits = std::max(1, (max_pages_per_seq + pps - 1) / pps);
  MTN_CHECK_ARG(max_splits <= 65535 * 32, "mtn_paged_decode: too many splits");
  const size_t need = mtn_paged_decode_workspace_bytes(n_seqs, num_q_heads, pool->num_kv_heads, D,
                                                       max_pages_per_seq, pps);
  if (max_splits > 1) {
    MTN_CHECK_ARG(workspace != nullptr && workspace_bytes >= need,
                  "mtn_paged_decode: workspace of %zu bytes < %zu needed", workspace_bytes, need);
    MTN_CHECK_ARG((reinterpret_cast<uintptr_t>(workspace) & 15) == 0, "mtn_paged_decode: workspace alignment");
  }

  mtn::DecodeParams prm{};
  const int64_t page_elems = static_cast<int64_t>(pool->num_kv_heads) * pool->page_size * D;
  auto* base = static_cast<const __nv_bfloat16*>(pool->base);
  prm.kpool = base + (static_cast<int64_t>(layer) * 2 + 0) * pool->num_pages * page_elems;
  prm.vpool = base + (static_cast<int64_t>(layer) * 2 + 1) * pool->num_pages * page_elems;
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
    case 64: return mtn::dispatch_nrep<64>(nrep, prm, n_seqs, s);
    case 128: return mtn::dispatch_nrep<128>(nrep, prm, n_seqs, s);
    default: return mtn::dispatch_nrep<256>(nrep, prm, n_seqs, s);
  }
}

}  // extern "C"
