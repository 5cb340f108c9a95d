// Fused CSA / HCA decode over a paged TurboQuant KV cache (sm_100a).
//
// One thread-block cluster of CS CTAs serves one query (one sequence, one
// decode step, one attention layer, all heads).  Reference semantics:
//
//   indexer   score[s] = sum_h softplus(w_h) * relu(q_h . k_s)
//             (aether_2b/modeling.py:609-615; decode data flow
//             aether_2b/serving.py:605-621, with the softplus of modeling.py)
//   top-k     exact top min(top_k, nb) by (score desc, index asc)
//   attention softmax over [selected compressed entries ; sliding window]
//             plus a per-head sink logit, K == V
//             (aether_pipeline/serving.py:99-130, modeling.py:158-178)
//   dequant   decode(c) = diag * WHT(c * s)   (aether_2b/turbo_quant.py:168-211)
//
// The cache stores y = WHT(diag * x) codes.  Because the normalised WHT is
// symmetric and orthogonal, q . decode(c) = s * (WHT(diag * q) . c): the
// kernel rotates each query once and works on the codes directly, keeps the
// weighted sum of the compressed values in the rotated domain, and applies
// one inverse WHT per head at the end.  The bf16 sliding window is not
// rotated and is accumulated separately.
//
// Phases of one CTA (rank r of the cluster):
//   1. TMA bulk copies stream this CTA's share of the query's index pages
//      (page table -> pool) into a shared-memory ring; the window rows are
//      fetched the same way.
//   2. Index scores on the tensor cores: the rotated index query is
//      quantised to 24-bit fixed point and split into three signed 8-bit
//      limbs, so mma.sync.s8 computes the code dot products exactly in
//      int32; one fp32 rounding combines the limbs.
//   3. Cluster-wide exact top-k: MSB-first 8-bit radix select over the
//      score bit patterns, histograms exchanged through distributed shared
//      memory; ties at the threshold go to the lowest block indices.  The
//      winners are compacted in ascending index order and pushed to the CTA
//      that attends them.
//   4. Each CTA gathers its slice of the selected rows (cp.async), expands
//      the codes to fp16 and runs QK^T / PV on mma.sync.f16 together with
//      its slice of the window; partial (max, sum, O_rot, O_win) per head
//      are pushed to the head's owner CTA, which merges them by log-sum-exp
//      with the sink, applies the inverse WHT and writes bf16.
//
// The HCA variant (modeling.py:384-410, serving.py:507-522) skips phases 2-3
// and attends every visible block.
#include <cooperative_groups.h>

#include "aether_b200.h"
#include "capi_util.cuh"
#include "common.cuh"

namespace cg = cooperative_groups;

namespace aether {

// profiling aid: the phase-timestamp buffer set by
// aether_csa_decode_set_debug_timer (null when off)
long long* cta_debug_buffer();

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRowH = kHeadDim + 8;  // fp16 row stride (halves) of MMA operand tiles: 272 B, conflict-free ldmatrix

template <int BITS, int CS, bool HCA>
struct CsaCfg {
  static constexpr int RB_IDX = kIdxDim * BITS / 8;   // bytes per index entry
  static constexpr int RB_KV = kHeadDim * BITS / 8;   // bytes per main entry
  // index pages per ring stage: ~36 KB stages (18 KB for 8-CTA clusters)
  static constexpr int CH = (CS >= 8 ? 8 : 16) / (BITS == 8 ? 2 : 1);
  static constexpr int STAGES = 2;
  static constexpr int MAX_KEYS = HCA ? 0 : (CS >= 8 ? 1024 : 2048);  // scored keys per CTA
  // compressed rows attended per CTA (max): the top-k slice, or for HCA a
  // contiguous range of visible blocks
  static constexpr int SELM = HCA ? 128 : ((256 / CS) < 16 ? 16 : (256 / CS));
  static constexpr int WINM = (128 / CS) < 16 ? 16 : (128 / CS);  // window rows per CTA (max)
  static constexpr int COLS = SELM + WINM;
  static constexpr int HPC = (kMaxHeads + CS - 1) / CS;  // heads merged per owner CTA (max)
  static constexpr int PST = COLS + 8;                     // P row stride (halves)

  // ---- shared memory layout (bytes) ----
  static constexpr int PB_IDX = page_bytes(RB_IDX);   // one index page: codes + scales
  static constexpr int PB_KV = page_bytes(RB_KV);
  static constexpr int STAGE_BYTES = CH * PB_IDX;
  static constexpr int RING = HCA ? 0 : STAGES * STAGE_BYTES;
  // attention-phase buffers alias the ring (it is dead once scoring ends)
  static constexpr int A_KC = 0;                                   // fp16 [SELM][kRowH]
  static constexpr int A_KW = A_KC + SELM * kRowH * 2;             // fp16 [WINM][kRowH]
  static constexpr int A_QR = A_KW + WINM * kRowH * 2;             // fp16 [16][kRowH]
  static constexpr int A_QW = A_QR + 16 * kRowH * 2;               // fp16 [16][kRowH]
  static constexpr int A_RAW = A_QW + 16 * kRowH * 2;              // codes [SELM][RB_KV]
  static constexpr int A_KS = A_RAW + SELM * RB_KV;                // fp32 [SELM]
  static constexpr int A_LOG = A_KS + SELM * 4;                    // fp32 [16][COLS]
  static constexpr int A_P = A_LOG + 16 * COLS * 4;                // fp16 [16][PST]
  static constexpr int A_END = (A_P + 16 * PST * 2 + 127) & ~127;
  static constexpr int REGION0 = RING > A_END ? RING : A_END;

  static constexpr int OFF_SCORES = REGION0;                       // u32 [MAX_KEYS]
  static constexpr int OFF_WIN = OFF_SCORES + MAX_KEYS * 4;        // bf16 [WINM][128]
  static constexpr int OFF_MERGE = OFF_WIN + WINM * kHeadDim * 2;  // fp32 [CS][HPC][MERGE_SLOT]
  static constexpr int MERGE_SLOT = 4 + 2 * kHeadDim;              // m, l, pad, pad, O_rot, O_win
  static constexpr int OFF_HIST = OFF_MERGE + CS * HPC * MERGE_SLOT * 4;  // u32 [2][256]
  static constexpr int OFF_SEL = OFF_HIST + 2 * 256 * 4;           // i32 [SELM]
  static constexpr int OFF_MISC = OFF_SEL + SELM * 4;              // small scalars
  static constexpr int MISC_BYTES = 1024;
  static constexpr int OFF_BAR = OFF_MISC + MISC_BYTES;            // mbarriers
  static constexpr int SMEM = OFF_BAR + 8 * (STAGES + 1);
  static_assert(CS * HPC * MERGE_SLOT * 4 >= kIdxHeads * kIdxDim * 4, "index-query scratch fits in merge area");
};

struct CsaParams {
  const __nv_bfloat16* q;       // [B, H, 128]
  const float* index_q;         // [B, 4, 64]
  const float* index_w;         // [B, 4]  raw head weights (softplus applied here)
  const float* sink;            // [H]
  const __nv_bfloat16* window;  // [B, W, 128]
  const int32_t* window_len;    // [B]
  const uint8_t* idx_pages;     // [P][64 x 64*bits/8 codes | 64 x fp32 scales]
  const uint8_t* kv_pages;      // [P][64 x 128*bits/8 codes | 64 x fp32 scales]
  const int32_t* page_table;    // [B, table_stride]
  const int32_t* nblocks;       // [B] visible compressed blocks
  const float* diag_idx;        // [64]  +-1
  const float* diag_kv;         // [128] +-1
  __nv_bfloat16* out;           // [B, H, 128]
  int32_t* sel_out;             // [B, top_k] or null
  float* score_out;             // [B, score_stride] index scores, or null
  int score_stride;
  long long* dbg;  // per-CTA phase timestamps [grid][16] (profiling aid), or null
  int* err;
  int table_stride, num_pages, H, W, top_k;
  float softmax_scale;
};

struct Misc {
  float alpha[kIdxHeads];
  float qscale[kIdxHeads];
  uint32_t strict[8];
  uint32_t eqc[8];
  int bstar;
  uint32_t above;
  uint32_t cnt_bin;
  uint32_t wsum[kWarps];
  float m_h[kMaxHeads];
  float l_h[kMaxHeads];
};

__device__ __forceinline__ uint32_t* remote_u32(cg::cluster_group& cl, uint32_t* p, int rank) {
  return cl.map_shared_rank(p, rank);
}

// Quantise x to the 24-bit fixed-point integer whose three signed 8-bit limbs
// (x = l2*65536 + l1*256 + l0) are returned.
__device__ __forceinline__ void limbs24(float x, float inv_unused, float s, int& l0, int& l1, int& l2) {
  int v = __float2int_rn(__fdiv_rn(x, s));
  l0 = ((v + 128) & 255) - 128;
  int v1 = (v - l0) >> 8;
  l1 = ((v1 + 128) & 255) - 128;
  l2 = (v1 - l1) >> 8;
}

template <int BITS>
__device__ __forceinline__ int phys_dim(int j, int h, int t, int e) {
  return BITS == 4 ? 16 * t + 8 * j + 2 * e + h : 16 * t + 8 * j + 4 * h + e;
}

template <int BITS, int CS, bool HCA>
__global__ void __launch_bounds__(kThreads) csa_decode_kernel(CsaParams p) {
  using C = CsaCfg<BITS, CS, HCA>;
  extern __shared__ __align__(128) uint8_t smem[];
  cg::cluster_group cl = cg::this_cluster();
  const int r = static_cast<int>(cl.block_rank());
  const int b = blockIdx.x / CS;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  auto stamp = [&](int slot) {  // SM clock cycles (phase durations)
    if (p.dbg && tid == 0) p.dbg[blockIdx.x * 16 + slot] = clock64();
  };
  stamp(0);

  uint32_t* scores = reinterpret_cast<uint32_t*>(smem + C::OFF_SCORES);
  __nv_bfloat16* winraw = reinterpret_cast<__nv_bfloat16*>(smem + C::OFF_WIN);
  float* merge = reinterpret_cast<float*>(smem + C::OFF_MERGE);
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem + C::OFF_HIST);
  int32_t* sel = reinterpret_cast<int32_t*>(smem + C::OFF_SEL);
  Misc* misc = reinterpret_cast<Misc*>(smem + C::OFF_MISC);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);

  // ------------------------------------------------------------ setup
  int nb = p.nblocks[b];
  const int max_nb = HCA ? CS * C::SELM : CS * C::MAX_KEYS;
  if (nb > max_nb || nb > p.table_stride * kPage) {
    if (tid == 0) report_error(p.err, kErrBadShape);
    nb = min(max_nb, p.table_stride * kPage);
  }
  if (nb < 0) nb = 0;
  const int K = HCA ? nb : min(p.top_k, nb);
  const int npages = (nb + kPage - 1) / kPage;
  const int ppc = (npages + CS - 1) / CS;
  const int pg0 = min(r * ppc, npages), pg1 = min(pg0 + ppc, npages);
  const int key0 = pg0 * kPage;
  const int nkeys = max(0, min(pg1 * kPage, nb) - key0);
  const int nchunks = (pg1 - pg0 + C::CH - 1) / C::CH;
  const int W = p.W;
  const int wpc = (W + CS - 1) / CS;
  int wl = p.window_len[b];
  wl = max(0, min(wl, W));
  const int wrow0 = r * wpc;
  const int wcnt = max(0, min(wl - wrow0, wpc));
  const int32_t* ptab = p.page_table + static_cast<long long>(b) * p.table_stride;

  if (tid == 0) {
    for (int i = 0; i < C::STAGES + 1; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  __syncthreads();

  auto issue_chunk = [&](int c) {
    const int stage = c % C::STAGES;
    uint8_t* dst = smem + stage * C::STAGE_BYTES;
    const int np = min(C::CH, pg1 - pg0 - c * C::CH);
    mbar_expect_tx(&bars[stage], np * C::PB_IDX);
    for (int i = 0; i < np; ++i) {
      int phys = ptab[pg0 + c * C::CH + i];
      if (phys < 0 || phys >= p.num_pages) {
        report_error(p.err, kErrBadPage);
        phys = 0;
      }
      bulk_g2s(dst + i * C::PB_IDX, p.idx_pages + static_cast<long long>(phys) * C::PB_IDX, C::PB_IDX, &bars[stage]);
    }
  };

  if (tid == 0) {
    if (wcnt > 0) {
      mbar_expect_tx(&bars[C::STAGES], wcnt * kHeadDim * 2);
      bulk_g2s(winraw, p.window + (static_cast<long long>(b) * W + wrow0) * kHeadDim, wcnt * kHeadDim * 2,
               &bars[C::STAGES]);
    }
    if (!HCA)
      for (int c = 0; c < min(nchunks, C::STAGES); ++c) issue_chunk(c);
  }

  int own_cnt = 0;  // selected rows this CTA attends
  int selp = 0;     // slice width of the selected list per CTA

  if (!HCA) {
    // -------------------------------------------------- index query prep
    // rotated index query q~_h = WHT(diag * q_h) (fp32), per-head 24-bit
    // fixed-point scale, alpha_h = softplus(w_h) * scale_h.
    float* qi = reinterpret_cast<float*>(smem + C::OFF_MERGE);  // [4][64] scratch, merge area unused yet
    if (warp < kIdxHeads) {
      const float* src = p.index_q + (static_cast<long long>(b) * kIdxHeads + warp) * kIdxDim;
      float v[2];
      v[0] = src[lane * 2] * p.diag_idx[lane * 2];
      v[1] = src[lane * 2 + 1] * p.diag_idx[lane * 2 + 1];
      // normalised WHT, 64 points, 2 per lane
#pragma unroll
      for (int h = 1; h < 64; h <<= 1) {
        if (h < 2) {
          float a = v[0], c2 = v[1];
          v[0] = a + c2;
          v[1] = a - c2;
        } else {
          const int ld = h / 2;
          const bool up = (lane & ld) != 0;
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            float o = __shfl_xor_sync(0xffffffffu, v[k], ld);
            v[k] = up ? o - v[k] : v[k] + o;
          }
        }
      }
      v[0] *= 0.125f;
      v[1] *= 0.125f;
      qi[warp * kIdxDim + lane * 2] = v[0];
      qi[warp * kIdxDim + lane * 2 + 1] = v[1];
      float am = warp_max(fmaxf(fabsf(v[0]), fabsf(v[1])));
      if (lane == 0) {
        float s = am > 0.f ? am / 8355000.0f : 1.0f;
        misc->qscale[warp] = s;
        misc->alpha[warp] = softplus_f(p.index_w[b * kIdxHeads + warp]) * s;
      }
    }
    __syncthreads();

    // B fragments: column n = g of n-tile 0 holds (head g/2, limb g%2), of
    // n-tile 1 (head g/2, limb 2) for even g and zero for odd g.
    uint32_t bq[2][2][2];
    {
      const int hq = g >> 1;
      const float s = misc->qscale[hq];
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t w0 = 0, w1 = 0;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int d = phys_dim<BITS>(j, hh, t, e);
            int l0, l1, l2;
            limbs24(qi[hq * kIdxDim + d], 0.f, s, l0, l1, l2);
            const int lA = (g & 1) ? l1 : l0;
            const int lB = (g & 1) ? 0 : l2;
            w0 |= (static_cast<uint32_t>(lA) & 0xFFu) << (8 * e);
            w1 |= (static_cast<uint32_t>(lB) & 0xFFu) << (8 * e);
          }
          bq[0][j][hh] = w0;
          bq[1][j][hh] = w1;
        }
    }
    float alpha_t = misc->alpha[t];

    // ------------------------------------------------------- scoring
    for (int c = 0; c < nchunks; ++c) {
      const int stage = c % C::STAGES;
      mbar_wait(&bars[stage], (c / C::STAGES) & 1, p.err);
      const uint8_t* stg = smem + stage * C::STAGE_BYTES;
      const int np = min(C::CH, pg1 - pg0 - c * C::CH);
      const int tiles = np * (kPage / 16);
      for (int tile = warp; tile < tiles; tile += kWarps) {
        const int rowA = tile * 16 + g, rowB = rowA + 8;  // rows within the stage
        const uint8_t* codes = stg + (tile >> 2) * C::PB_IDX;  // the tile's page
        const float* ksc = reinterpret_cast<const float*>(codes + kPage * C::RB_IDX);
        const int ra = rowA & 63, rbb = rowB & 63;
        uint32_t a[2][4];
        if (BITS == 4) {
          const uint2 va = *reinterpret_cast<const uint2*>(codes + ra * C::RB_IDX + t * 8);
          const uint2 vb = *reinterpret_cast<const uint2*>(codes + rbb * C::RB_IDX + t * 8);
          uint32_t la0, ha0, la1, ha1, lb0, hb0, lb1, hb1;
          nib_to_s8(va.x, la0, ha0);
          nib_to_s8(va.y, la1, ha1);
          nib_to_s8(vb.x, lb0, hb0);
          nib_to_s8(vb.y, lb1, hb1);
          a[0][0] = la0; a[0][1] = lb0; a[0][2] = ha0; a[0][3] = hb0;
          a[1][0] = la1; a[1][1] = lb1; a[1][2] = ha1; a[1][3] = hb1;
        } else {
          const uint4 va = *reinterpret_cast<const uint4*>(codes + ra * C::RB_IDX + t * 16);
          const uint4 vb = *reinterpret_cast<const uint4*>(codes + rbb * C::RB_IDX + t * 16);
          a[0][0] = va.x; a[0][1] = vb.x; a[0][2] = va.y; a[0][3] = vb.y;
          a[1][0] = va.z; a[1][1] = vb.z; a[1][2] = va.w; a[1][3] = vb.w;
        }
        int acc0[4] = {0, 0, 0, 0}, acc1[4] = {0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          mma_s8(acc0, a[j][0], a[j][1], a[j][2], a[j][3], bq[0][j][0], bq[0][j][1]);
          mma_s8(acc1, a[j][0], a[j][1], a[j][2], a[j][3], bq[1][j][0], bq[1][j][1]);
        }
        // thread t holds head t: limbs (acc0[0], acc0[1], acc1[0]) for row A,
        // (acc0[2], acc0[3], acc1[2]) for row B.
        const float dA = __fadd_rn(__fmul_rn(static_cast<float>(acc1[0]), 65536.f),
                                   __fadd_rn(__fmul_rn(static_cast<float>(acc0[1]), 256.f),
                                             static_cast<float>(acc0[0])));
        const float dB = __fadd_rn(__fmul_rn(static_cast<float>(acc1[2]), 65536.f),
                                   __fadd_rn(__fmul_rn(static_cast<float>(acc0[3]), 256.f),
                                             static_cast<float>(acc0[2])));
        float sA = alpha_t * fmaxf(dA, 0.f);
        float sB = alpha_t * fmaxf(dB, 0.f);
        sA += __shfl_xor_sync(0xffffffffu, sA, 1);
        sB += __shfl_xor_sync(0xffffffffu, sB, 1);
        sA += __shfl_xor_sync(0xffffffffu, sA, 2);
        sB += __shfl_xor_sync(0xffffffffu, sB, 2);
        const int lrow = t == 0 ? rowA : rowB;
        if (t < 2) {
          const int key = c * C::CH * kPage + lrow;  // CTA-local key index
          if (key < nkeys) {
            float s = __fadd_rn(__fmul_rn(t == 0 ? sA : sB, ksc[lrow & 63]), 0.0f);
            scores[key] = __float_as_uint(s) + 1u;
          }
        }
      }
      __syncthreads();
      if (tid == 0 && c + C::STAGES < nchunks) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        issue_chunk(c + C::STAGES);
      }
    }

    if (p.score_out) {
      float* so = p.score_out + static_cast<long long>(b) * p.score_stride + key0;
      for (int i = tid; i < nkeys; i += kThreads) so[i] = __uint_as_float(scores[i] - 1u);
    }

    // ------------------------------------------- cluster radix select
    uint32_t prefix = 0;
    int nbits = 0;
    bool all_eq = true;
    uint32_t R = static_cast<uint32_t>(K);
    if (tid < 8) {
      misc->strict[tid] = 0;
      misc->eqc[tid] = 0;
    }
    if (nb > K) {
      all_eq = false;
      for (int pass = 0; pass < 4; ++pass) {
        uint32_t* h = hist + (pass & 1) * 256;
        h[tid] = 0;
        __syncthreads();
        const int shift = 24 - 8 * pass;
        for (int base = 0; base < nkeys; base += kThreads) {
          const int i = base + tid;
          bool m = false;
          uint32_t dig = 0xFFFFFFFFu;
          if (i < nkeys) {
            const uint32_t key = scores[i];
            m = nbits == 0 || (key >> (32 - nbits)) == prefix;
            if (m) dig = (key >> shift) & 255u;
          }
          if (m) atomicAdd(&h[dig], 1u);
        }
        cl.sync();
        uint32_t cnt[CS];
        uint32_t tot = 0;
#pragma unroll
        for (int rr = 0; rr < CS; ++rr) {
          cnt[rr] = *remote_u32(cl, h + tid, rr);
          tot += cnt[rr];
        }
        // descending-bin scan in warp 0 over per-thread totals staged in
        // the other histogram buffer (its previous contents are dead).
        uint32_t* tots = hist + ((pass + 1) & 1) * 256;
        // The other buffer may still be read remotely for pass-1 data?  No:
        // every CTA finished reading pass-1 histograms before arriving at
        // this pass's cluster barrier.
        tots[tid] = tot;
        __syncthreads();
        if (warp == 0) {
          uint32_t s8 = 0;
#pragma unroll
          for (int k = 0; k < 8; ++k) s8 += tots[255 - 8 * lane - k];
          uint32_t inc = s8;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            uint32_t v = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += v;
          }
          const uint32_t exc = inc - s8;
          const bool hit = exc < R && inc >= R;
          const uint32_t hm = __ballot_sync(0xffffffffu, hit);
          if (hit && lane == __ffs(hm) - 1) {
            uint32_t cum = exc;
            for (int k = 0; k < 8; ++k) {
              const int bin = 255 - 8 * lane - k;
              const uint32_t v = tots[bin];
              if (cum + v >= R) {
                misc->bstar = bin;
                misc->above = cum;
                misc->cnt_bin = v;
                break;
              }
              cum += v;
            }
          }
        }
        __syncthreads();
        const int bs = misc->bstar;
        // per-rank counts strictly above the chosen bin, and in it
#pragma unroll
        for (int rr = 0; rr < CS; ++rr) {
          uint32_t v = tid > bs ? cnt[rr] : 0u;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
          if (lane == 0 && v) atomicAdd(&misc->strict[rr], v);
          if (tid == bs) misc->eqc[rr] = cnt[rr];
        }
        R -= misc->above;
        prefix = (prefix << 8) | static_cast<uint32_t>(bs);
        nbits += 8;
        const bool done = misc->cnt_bin == R;
        __syncthreads();
        if (done) {
          all_eq = true;
          break;
        }
      }
    } else {
      // every visible block is selected
      if (tid < CS) {
        const int rp0 = min(tid * ppc, npages), rp1 = min(rp0 + ppc, npages);
        misc->eqc[tid] = max(0, min(rp1 * kPage, nb) - rp0 * kPage);
      }
      cl.sync();  // all CTAs of the cluster are running before remote stores
    }
    __syncthreads();

    // ------------------------------------ ordered compaction and push
    selp = (((K + CS - 1) / CS) + 15) & ~15;
    uint32_t take[CS], off[CS];
    {
      uint32_t eq_before = 0, sel_before = 0;
#pragma unroll
      for (int rr = 0; rr < CS; ++rr) {
        const uint32_t e = misc->eqc[rr];
        uint32_t tk = e;
        if (!all_eq) tk = R > eq_before ? min(e, R - eq_before) : 0u;
        take[rr] = tk;
        off[rr] = sel_before;
        sel_before += misc->strict[rr] + tk;
        eq_before += e;
      }
    }
    const int E = (nkeys + kThreads - 1) / kThreads;
    const int i0 = min(tid * E, nkeys), i1 = min(i0 + E, nkeys);
    uint32_t cs = 0, ce = 0;
    for (int i = i0; i < i1; ++i) {
      const uint32_t top = nbits ? (scores[i] >> (32 - nbits)) : 0u;
      if (top > prefix) ++cs;
      else if (top == prefix) ++ce;
    }
    uint32_t packed = cs | (ce << 16);
    uint32_t inc = packed;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      uint32_t v = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += v;
    }
    if (lane == 31) misc->wsum[warp] = inc;
    __syncthreads();
    uint32_t wbase = 0;
    for (int w = 0; w < warp; ++w) wbase += misc->wsum[w];
    uint32_t exc = wbase + inc - packed;
    uint32_t sb = exc & 0xFFFFu, eb = exc >> 16;
    uint32_t my_take = 0, my_off = 0;
#pragma unroll
    for (int rr = 0; rr < CS; ++rr)
      if (rr == r) {
        my_take = take[rr];
        my_off = off[rr];
      }
    for (int i = i0; i < i1; ++i) {
      const uint32_t top = nbits ? (scores[i] >> (32 - nbits)) : 0u;
      int pos = -1;
      if (top > prefix) {
        pos = static_cast<int>(my_off + sb + min(eb, my_take));
        ++sb;
      } else if (top == prefix) {
        if (eb < my_take) pos = static_cast<int>(my_off + sb + eb);
        ++eb;
      }
      if (pos >= 0 && pos < K) {
        const int owner = pos / selp;
        int32_t* dst = cl.map_shared_rank(sel, owner);
        dst[pos - owner * selp] = key0 + i;
      }
    }
    cl.sync();
    own_cnt = max(0, min(K - r * selp, selp));
    if (p.sel_out) {
      int32_t* so = p.sel_out + static_cast<long long>(b) * p.top_k;
      for (int i = tid; i < own_cnt; i += kThreads) so[r * selp + i] = sel[i];
      for (int i = K + r + CS * tid; i < p.top_k; i += CS * kThreads) so[i] = -1;
    }
  } else {
    // HCA: attend every visible block; CTA r takes a contiguous range.
    selp = (((K + CS - 1) / CS) + 15) & ~15;
    own_cnt = max(0, min(K - r * selp, selp));
    for (int i = tid; i < own_cnt; i += kThreads) sel[i] = r * selp + i;
    cl.sync();  // all CTAs running before remote stores in the merge
  }
  stamp(1);

  // =============================================== attention (this slice)
  __half* Kc = reinterpret_cast<__half*>(smem + C::A_KC);
  __half* Kw = reinterpret_cast<__half*>(smem + C::A_KW);
  __half* Qr = reinterpret_cast<__half*>(smem + C::A_QR);
  __half* Qw = reinterpret_cast<__half*>(smem + C::A_QW);
  uint8_t* raw = smem + C::A_RAW;
  float* ks = reinterpret_cast<float*>(smem + C::A_KS);
  float* logit = reinterpret_cast<float*>(smem + C::A_LOG);
  __half* P = reinterpret_cast<__half*>(smem + C::A_P);
  __syncthreads();

  // gather the selected main rows of this slice
  {
    constexpr int CPR = C::RB_KV / 16;  // 16-byte chunks per row
    for (int i = tid; i < own_cnt * CPR; i += kThreads) {
      const int row = i / CPR, ch = i % CPR;
      const int blk = sel[row];
      int phys = ptab[blk >> 6];
      if (phys < 0 || phys >= p.num_pages) {
        report_error(p.err, kErrBadPage);
        phys = 0;
      }
      const uint8_t* pg = p.kv_pages + static_cast<long long>(phys) * C::PB_KV;
      cp_async16(raw + row * C::RB_KV + ch * 16, pg + (blk & 63) * C::RB_KV + ch * 16);
      if (ch == 0) cp_async4(ks + row, pg + kPage * C::RB_KV + (blk & 63) * 4);
    }
  }
  // queries: plain (for the window) and rotated WHT(diag * q) (for the codes)
  for (int h = warp; h < kMaxHeads; h += kWarps) {
    float v[4];
    if (h < p.H) {
      const __nv_bfloat16* src = p.q + (static_cast<long long>(b) * p.H + h) * kHeadDim + lane * 4;
#pragma unroll
      for (int k = 0; k < 4; ++k) v[k] = __bfloat162float(src[k]);
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) v[k] = 0.f;
    }
    __half* qw = Qw + h * kRowH + lane * 4;
    *reinterpret_cast<uint2*>(qw) = make_uint2(pack_half2(v[0], v[1]), pack_half2(v[2], v[3]));
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] *= p.diag_kv[lane * 4 + k];
#pragma unroll
    for (int hs = 1; hs < kHeadDim; hs <<= 1) {
      if (hs < 4) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if ((k & hs) == 0) {
            float a = v[k], c2 = v[k + hs];
            v[k] = a + c2;
            v[k + hs] = a - c2;
          }
      } else {
        const int ld = hs / 4;
        const bool up = (lane & ld) != 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float o = __shfl_xor_sync(0xffffffffu, v[k], ld);
          v[k] = up ? o - v[k] : v[k] + o;
        }
      }
    }
    const float cn = 0.0883883461356163f;
    __half* qr = Qr + h * kRowH + lane * 4;
    *reinterpret_cast<uint2*>(qr) =
        make_uint2(pack_half2(v[0] * cn, v[1] * cn), pack_half2(v[2] * cn, v[3] * cn));
  }
  stamp(2);
  // window rows -> fp16 tiles (rows beyond wcnt zero-filled to the tile edge)
  const int ntw = (wcnt + 15) / 16;
  if (wcnt > 0) mbar_wait(&bars[C::STAGES], 0, p.err);
  for (int i = tid; i < ntw * 16 * (kHeadDim / 8); i += kThreads) {
    const int row = i / (kHeadDim / 8), c8 = (i % (kHeadDim / 8)) * 8;
    uint4 o = make_uint4(0, 0, 0, 0);
    if (row < wcnt) {
      const uint4 v = *reinterpret_cast<const uint4*>(winraw + row * kHeadDim + c8);
      const __nv_bfloat162* bv = reinterpret_cast<const __nv_bfloat162*>(&v);
      float2 f0 = __bfloat1622float2(bv[0]), f1 = __bfloat1622float2(bv[1]);
      float2 f2 = __bfloat1622float2(bv[2]), f3 = __bfloat1622float2(bv[3]);
      o = make_uint4(pack_half2(f0.x, f0.y), pack_half2(f1.x, f1.y), pack_half2(f2.x, f2.y),
                     pack_half2(f3.x, f3.y));
    }
    *reinterpret_cast<uint4*>(Kw + row * kRowH + c8) = o;
  }
  cp_async_commit_wait_all();
  __syncthreads();
  stamp(3);
  // codes -> exact fp16 integers
  const int ntc = (own_cnt + 15) / 16;
  for (int i = tid; i < ntc * 16 * (kHeadDim / 8); i += kThreads) {
    const int row = i / (kHeadDim / 8), c8 = (i % (kHeadDim / 8)) * 8;
    uint4 o = make_uint4(0, 0, 0, 0);
    if (row < own_cnt) {
      float f[8];
      if (BITS == 8) {
        const uint2 v = *reinterpret_cast<const uint2*>(raw + row * C::RB_KV + c8);
        const int8_t* cb = reinterpret_cast<const int8_t*>(&v);
#pragma unroll
        for (int k = 0; k < 8; ++k) f[k] = static_cast<float>(cb[k]);
      } else {
        const uint32_t v = *reinterpret_cast<const uint32_t*>(raw + row * C::RB_KV + c8 / 2);
        uint32_t lo, hi;
        nib_to_s8(v, lo, hi);
        const int8_t* lb = reinterpret_cast<const int8_t*>(&lo);
        const int8_t* hb = reinterpret_cast<const int8_t*>(&hi);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          f[2 * k] = static_cast<float>(lb[k]);
          f[2 * k + 1] = static_cast<float>(hb[k]);
        }
      }
      o = make_uint4(pack_half2(f[0], f[1]), pack_half2(f[2], f[3]), pack_half2(f[4], f[5]),
                     pack_half2(f[6], f[7]));
    }
    *reinterpret_cast<uint4*>(Kc + row * kRowH + c8) = o;
  }
  __syncthreads();

  stamp(4);
  // ---- S = Q K^T per 16-source tile (compressed tiles first, then window)
  const int ncols_c = ntc * 16;
  const int ncols = ncols_c + ntw * 16;
  for (int tile = warp; tile < ntc + ntw; tile += kWarps) {
    const bool comp = tile < ntc;
    const __half* Q = comp ? Qr : Qw;
    const __half* Kt = comp ? Kc + tile * 16 * kRowH : Kw + (tile - ntc) * 16 * kRowH;
    float acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll
    for (int kk = 0; kk < kHeadDim / 16; ++kk) {
      uint32_t a[4];
      ldsm_x4(a[0], a[1], a[2], a[3], Q + (lane & 15) * kRowH + kk * 16 + (lane >> 4) * 8);
      uint32_t b0, b1, b2, b3;
      ldsm_x4(b0, b1, b2, b3, Kt + ((lane & 7) + ((lane >> 4) << 3)) * kRowH + kk * 16 + ((lane >> 3) & 1) * 8);
      mma_f16(acc[0], a, b0, b1);
      mma_f16(acc[1], a, b2, b3);
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = g + (e >> 1) * 8;
        const int src = nt * 8 + 2 * t + (e & 1);  // within tile
        float z;
        if (comp) {
          const int row = tile * 16 + src;
          z = row < own_cnt ? acc[nt][e] * ks[row] * p.softmax_scale : -INFINITY;
        } else {
          const int row = (tile - ntc) * 16 + src;
          z = row < wcnt ? acc[nt][e] * p.softmax_scale : -INFINITY;
        }
        logit[h * C::COLS + tile * 16 + src] = z;
      }
  }
  __syncthreads();

  stamp(5);
  // ---- per-head max / exp / sum over this CTA's sources
  for (int h = warp; h < kMaxHeads; h += kWarps) {
    float m = -INFINITY;
    for (int c = lane; c < ncols; c += 32) m = fmaxf(m, logit[h * C::COLS + c]);
    m = warp_max(m);
    const float mu = m == -INFINITY ? 0.f : m;
    float l = 0.f;
    for (int c = lane; c < ncols; c += 32) {
      const float e = __expf(logit[h * C::COLS + c] - mu);
      l += e;
      const float w = c < ncols_c ? e * ks[c < own_cnt ? c : 0] : e;
      P[h * C::PST + c] = __float2half_rn(h < p.H ? w : 0.f);
    }
    l = warp_sum(l);
    if (lane == 0) {
      misc->m_h[h] = m;
      misc->l_h[h] = l;
    }
  }
  __syncthreads();

  // ---- O = P V: warp w owns output dims [16w, 16w+16)
  float orot[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}}, owin[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
  {
    const int d0 = warp * 16;
    for (int kt = 0; kt < ntc + ntw; ++kt) {
      const bool comp = kt < ntc;
      const __half* V = comp ? Kc + kt * 16 * kRowH : Kw + (kt - ntc) * 16 * kRowH;
      uint32_t a[4];
      ldsm_x4(a[0], a[1], a[2], a[3], P + (lane & 15) * C::PST + kt * 16 + (lane >> 4) * 8);
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(b0, b1, b2, b3, V + ((lane & 7) + ((lane >> 3) & 1) * 8) * kRowH + d0 + (lane >> 4) * 8);
      if (comp) {
        mma_f16(orot[0], a, b0, b1);
        mma_f16(orot[1], a, b2, b3);
      } else {
        mma_f16(owin[0], a, b0, b1);
        mma_f16(owin[1], a, b2, b3);
      }
    }
  }

  stamp(6);
  // ---- push partials to the owner CTA of each head
  const int hpc = (p.H + CS - 1) / CS;
#pragma unroll
  for (int e2 = 0; e2 < 2; ++e2) {
    const int h = g + e2 * 8;
    if (h < p.H) {
      const int owner = h / hpc, lh = h % hpc;
      float* slot = cl.map_shared_rank(merge, owner) + (r * C::HPC + lh) * C::MERGE_SLOT;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int d = warp * 16 + nt * 8 + 2 * t;
        *reinterpret_cast<float2*>(slot + 4 + d) = make_float2(orot[nt][e2 * 2], orot[nt][e2 * 2 + 1]);
        *reinterpret_cast<float2*>(slot + 4 + kHeadDim + d) = make_float2(owin[nt][e2 * 2], owin[nt][e2 * 2 + 1]);
      }
      if (warp == 0 && t == 0) {
        slot[0] = misc->m_h[h];
        slot[1] = misc->l_h[h];
      }
    }
  }
  cl.sync();
  stamp(7);

  // ---- owner: log-sum-exp merge with the sink, inverse WHT, bf16 store
  for (int lh = warp; lh < hpc; lh += kWarps) {
    const int h = r * hpc + lh;
    if (h >= p.H) break;
    const float sk = p.sink[h];
    float M = sk;
#pragma unroll
    for (int rr = 0; rr < CS; ++rr) M = fmaxf(M, merge[(rr * C::HPC + lh) * C::MERGE_SLOT]);
    float L = __expf(sk - M);
    float vr[4] = {0, 0, 0, 0}, vw[4] = {0, 0, 0, 0};
#pragma unroll
    for (int rr = 0; rr < CS; ++rr) {
      const float* slot = merge + (rr * C::HPC + lh) * C::MERGE_SLOT;
      const float m = slot[0];
      const float a = m == -INFINITY ? 0.f : __expf(m - M);
      L += a * slot[1];
      const float4 o1 = *reinterpret_cast<const float4*>(slot + 4 + lane * 4);
      const float4 o2 = *reinterpret_cast<const float4*>(slot + 4 + kHeadDim + lane * 4);
      vr[0] += a * o1.x; vr[1] += a * o1.y; vr[2] += a * o1.z; vr[3] += a * o1.w;
      vw[0] += a * o2.x; vw[1] += a * o2.y; vw[2] += a * o2.z; vw[3] += a * o2.w;
    }
    // inverse rotation of the compressed part: diag * WHT(v)
#pragma unroll
    for (int hs = 1; hs < kHeadDim; hs <<= 1) {
      if (hs < 4) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if ((k & hs) == 0) {
            float a = vr[k], c2 = vr[k + hs];
            vr[k] = a + c2;
            vr[k + hs] = a - c2;
          }
      } else {
        const int ld = hs / 4;
        const bool up = (lane & ld) != 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float o = __shfl_xor_sync(0xffffffffu, vr[k], ld);
          vr[k] = up ? o - vr[k] : vr[k] + o;
        }
      }
    }
    const float inv = 1.f / L;
    __nv_bfloat16* dst = p.out + (static_cast<long long>(b) * p.H + h) * kHeadDim + lane * 4;
    float o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
      o[k] = (vr[k] * 0.0883883461356163f * p.diag_kv[lane * 4 + k] + vw[k]) * inv;
    __nv_bfloat162 o01 = __floats2bfloat162_rn(o[0], o[1]), o23 = __floats2bfloat162_rn(o[2], o[3]);
    *reinterpret_cast<uint2*>(dst) =
        make_uint2(*reinterpret_cast<uint32_t*>(&o01), *reinterpret_cast<uint32_t*>(&o23));
  }
  stamp(8);
}

template <int BITS, int CS, bool HCA>
static int launch_csa(const CsaParams& p, int B, cudaStream_t st) {
  using C = CsaCfg<BITS, CS, HCA>;
  auto kern = csa_decode_kernel<BITS, CS, HCA>;
  if (int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), C::SMEM, "csa_decode")) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(B * CS);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CS;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  AETHER_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p), "csa_decode: launch");
  return 0;
}

template <bool HCA>
static int dispatch_csa(const CsaParams& p, int B, int bits, int cs, cudaStream_t st) {
  if (bits == 4 && cs == 4) return launch_csa<4, 4, HCA>(p, B, st);
  if (bits == 4 && cs == 8) return launch_csa<4, 8, HCA>(p, B, st);
  if (bits == 8 && cs == 4) return launch_csa<8, 4, HCA>(p, B, st);
  if (bits == 8 && cs == 8) return launch_csa<8, 8, HCA>(p, B, st);
  set_last_error("csa_decode: unsupported (bits=%d, cluster=%d)", bits, cs);
  return 1;
}

static int max_blocks_for(bool hca, int bits, int cs) {
  (void)bits;
  if (hca) return cs * 128;
  return cs * (cs >= 8 ? 1024 : 2048);
}

static int choose_cluster(int B, bool hca, int bits, int max_nblocks) {
  // Enough CTAs to cover the 148 SMs about twice; larger clusters when the
  // batch is small or the context long.
  int cs = (B * 4 >= 2 * 148) ? 4 : 8;
  if (max_nblocks > max_blocks_for(hca, bits, cs)) cs = 8;
  return cs;
}

static int csa_common(bool hca, const void* q, const float* index_q, const float* index_w, const float* sink,
                      const void* window, const int32_t* window_len, const uint8_t* idx_pages, const uint8_t* kv_pages,
                      const int32_t* page_table, int table_stride, int num_pages, const int32_t* nblocks,
                      int max_nblocks, const float* diag_idx, const float* diag_kv, int B, int H, int W, int bits,
                      int top_k, float softmax_scale, void* out, int32_t* sel_out, int* err, int cluster,
                      void* stream, float* score_out = nullptr, int score_stride = 0) {
  AETHER_REQUIRE(bits == 4 || bits == 8, "bits must be 4 or 8, got %d", bits);
  AETHER_REQUIRE(H >= 1 && H <= kMaxHeads, "num_heads must be in [1, %d], got %d", kMaxHeads, H);
  AETHER_REQUIRE(W >= 0 && W <= 128, "window capacity must be in [0, 128], got %d", W);
  AETHER_REQUIRE(B >= 0, "batch must be non-negative");
  AETHER_REQUIRE(table_stride >= 1 && num_pages >= 1, "page table / pool must be non-empty");
  if (!hca) AETHER_REQUIRE(top_k >= 1 && top_k <= 256, "top_k must be in [1, 256], got %d", top_k);
  int cs = cluster > 0 ? cluster : choose_cluster(B, hca, bits, max_nblocks);
  AETHER_REQUIRE(cs == 4 || cs == 8, "cluster size must be 4 or 8, got %d", cs);
  AETHER_REQUIRE(max_nblocks <= max_blocks_for(hca, bits, cs),
                 "%s decode: %d visible blocks exceed the single-cluster limit %d", hca ? "hca" : "csa",
                 max_nblocks, max_blocks_for(hca, bits, cs));
  if (B == 0) return 0;
  CsaParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.index_q = index_q;
  p.index_w = index_w;
  p.sink = sink;
  p.window = static_cast<const __nv_bfloat16*>(window);
  p.window_len = window_len;
  p.idx_pages = idx_pages;
  p.kv_pages = kv_pages;
  p.page_table = page_table;
  p.nblocks = nblocks;
  p.diag_idx = diag_idx;
  p.diag_kv = diag_kv;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.sel_out = sel_out;
  p.score_out = score_out;
  p.score_stride = score_stride;
  p.err = err;
  p.table_stride = table_stride;
  p.num_pages = num_pages;
  p.H = H;
  p.W = W;
  p.top_k = hca ? 0 : top_k;
  p.dbg = cta_debug_buffer();
  p.softmax_scale = softmax_scale;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = hca ? dispatch_csa<true>(p, B, bits, cs, st) : dispatch_csa<false>(p, B, bits, cs, st);
  if (rc) return rc;
  return check_launch(hca ? "hca_decode_paged" : "csa_decode_paged");
}

int hca_decode_cta(const void* q, const float* sink, const void* window, const int32_t* window_len,
                   const uint8_t* kv_pages, const int32_t* page_table, int table_stride, int num_pages,
                   const int32_t* nblocks, int max_nblocks, const float* diag_kv, int B, int H, int W, int bits,
                   float softmax_scale, void* out, int* err, int pdl, void* stream);
int csa_decode_cta(const void* q, const float* index_q, const float* index_w, const float* sink, const void* window,
                   const int32_t* window_len, const uint8_t* idx_pages, const uint8_t* kv_pages,
                   const int32_t* page_table, int table_stride, int num_pages, const int32_t* nblocks,
                   int max_nblocks, const float* diag_idx, const float* diag_kv, int B, int H, int W, int bits,
                   int top_k, float softmax_scale, void* out, int32_t* sel_out, float* score_out, int score_stride,
                   uint32_t* workspace, int* err, int pdl, void* stream,
                   const int32_t* rope_pos = nullptr, const float* rope_inv_freq = nullptr,
                   int rope_dim = 0, const uint32_t* step_flags = nullptr, uint32_t step_seq = 0);

}  // namespace aether

using namespace aether;

extern "C" {

int aether_csa_decode_paged(const void* q, const float* index_q, const float* index_w, const float* sink,
                            const void* window, const int32_t* window_len, const uint8_t* idx_pages, const uint8_t* kv_pages,
                            const int32_t* page_table, int table_stride, int num_pages, const int32_t* nblocks,
                            int max_nblocks, const float* diag_idx, const float* diag_kv, int B, int H, int W,
                            int bits, int top_k, float softmax_scale, void* out, int32_t* sel_out,
                            uint32_t* workspace, int* err, int cluster, int pdl, void* stream) {
  AETHER_REQUIRE(index_q && index_w && idx_pages && diag_idx, "csa_decode_paged: null index input");
  if (cluster <= 1)
    return csa_decode_cta(q, index_q, index_w, sink, window, window_len, idx_pages, kv_pages, page_table,
                          table_stride, num_pages, nblocks, max_nblocks, diag_idx, diag_kv, B, H, W, bits, top_k,
                          softmax_scale, out, sel_out, nullptr, 0, workspace, err, pdl, stream);
  return csa_common(false, q, index_q, index_w, sink, window, window_len, idx_pages, kv_pages,
                    page_table, table_stride, num_pages, nblocks, max_nblocks, diag_idx, diag_kv, B, H, W, bits,
                    top_k, softmax_scale, out, sel_out, err, cluster, stream);
}

// aether_csa_decode_paged (score + select/attend kernels) that also applies
// the inverse output RoPE: the last rope_dim channels of each head's output
// are rotated by -rope_pos[b] with rope_inv_freq [rope_dim / 2], as
// aether_2b/serving.py:469-472 does before the output projection.
int aether_csa_decode_paged_rope(const void* q, const float* index_q, const float* index_w, const float* sink,
                                 const void* window, const int32_t* window_len, const uint8_t* idx_pages,
                                 const uint8_t* kv_pages, const int32_t* page_table, int table_stride, int num_pages,
                                 const int32_t* nblocks, int max_nblocks, const float* diag_idx, const float* diag_kv,
                                 int B, int H, int W, int bits, int top_k, float softmax_scale, void* out,
                                 int32_t* sel_out, uint32_t* workspace, int* err, int pdl, const int32_t* rope_pos,
                                 const float* rope_inv_freq, int rope_dim, void* stream) {
  AETHER_REQUIRE(index_q && index_w && idx_pages && diag_idx, "csa_decode_paged: null index input");
  AETHER_REQUIRE(rope_inv_freq && rope_pos, "csa_decode_paged_rope: null RoPE input");
  return csa_decode_cta(q, index_q, index_w, sink, window, window_len, idx_pages, kv_pages, page_table, table_stride,
                        num_pages, nblocks, max_nblocks, diag_idx, diag_kv, B, H, W, bits, top_k, softmax_scale, out,
                        sel_out, nullptr, 0, workspace, err, pdl, stream, rope_pos, rope_inv_freq, rope_dim);
}

// aether_csa_decode_paged with host buffers: copies in_bytes of packed
// step inputs from (pinned) host_in to dev_in, runs the decode, and copies
// out_bytes of packed results from dev_out to (pinned) host_out, all
// enqueued by this one call.  The device pointers (q, index_q, ..., out,
// sel_out) point into dev_in / dev_out.  With h2d_stream / d2h_stream and the
// slot's three events (ev_h2d, ev_comp, ev_d2h) given, the input copy runs on
// h2d_stream after the slot's previous decode, the decode on `stream`, and the
// output copy on d2h_stream after the decode; alternating two slots (staging
// buffers and events) lets one step's copies overlap its neighbours' kernels.
// With them null everything runs on `stream` in order.
//
// How the decode waits for its copies: a stream wait on another stream's
// event in front of the score kernel also ends the programmatic (PDL)
// overlap with the previous step's attend kernel, which costs ~3.5 us per
// step.  With slot_flags (two device u32 words per staging slot, zero
// before the slot's first step) and seq (1, 2, 3, ... per slot, mod 2^32), the copy
// streams instead write seq into slot_flags[0] after the input copy and into
// slot_flags[1] after the output copy (stream memory operations), and the
// kernels poll them with bounded waits: the score kernel for this step's
// inputs, the attend kernel for the slot's previous output copy before its
// stores.  Without slot_flags, or where the driver lacks stream memory
// operations, the decode stream waits on ev_h2d and ev_d2h instead.
typedef int (*WriteValue32Fn)(cudaStream_t, unsigned long long, unsigned int, unsigned int);
static WriteValue32Fn write_value32() {
  static const WriteValue32Fn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuStreamWriteValue32", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      return static_cast<WriteValue32Fn>(nullptr);
    }
    return reinterpret_cast<WriteValue32Fn>(f);
  }();
  return fn;
}

static int write_seq(cudaStream_t s, uint32_t* word, uint32_t seq, const char* what) {
  const int rc = write_value32()(s, reinterpret_cast<unsigned long long>(word), seq, 0u);
  AETHER_REQUIRE(rc == 0, "csa_decode_paged_host: %s (driver error %d)", what, rc);
  return 0;
}

int aether_csa_decode_paged_host(const void* host_in, void* dev_in, size_t in_bytes, void* host_out,
                                 const void* dev_out, size_t out_bytes, const void* q, const float* index_q,
                                 const float* index_w, const float* sink, const void* window,
                                 const int32_t* window_len, const uint8_t* idx_pages, const uint8_t* kv_pages,
                                 const int32_t* page_table, int table_stride, int num_pages, const int32_t* nblocks,
                                 int max_nblocks, const float* diag_idx, const float* diag_kv, int B, int H, int W,
                                 int bits, int top_k, float softmax_scale, void* out, int32_t* sel_out,
                                 uint32_t* workspace, int* err, int pdl, void* stream, void* h2d_stream,
                                 void* d2h_stream, void* ev_h2d, void* ev_comp, void* ev_d2h, uint32_t* slot_flags,
                                 uint32_t seq) {
  AETHER_REQUIRE(host_in && dev_in && host_out && dev_out, "csa_decode_paged_host: null buffer");
  AETHER_REQUIRE(index_q && index_w && idx_pages && diag_idx, "csa_decode_paged: null index input");
  const bool split = h2d_stream != nullptr;
  AETHER_REQUIRE(!split || (d2h_stream && ev_h2d && ev_comp && ev_d2h),
                 "csa_decode_paged_host: copy streams need d2h_stream and the slot's three events");
  AETHER_REQUIRE(!slot_flags || split, "csa_decode_paged_host: slot flags need copy streams");
  const bool flags = slot_flags != nullptr && write_value32() != nullptr;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaStream_t sin = split ? static_cast<cudaStream_t>(h2d_stream) : st;
  cudaStream_t sout = split ? static_cast<cudaStream_t>(d2h_stream) : st;
  cudaEvent_t eh = static_cast<cudaEvent_t>(ev_h2d), ec = static_cast<cudaEvent_t>(ev_comp),
              ed = static_cast<cudaEvent_t>(ev_d2h);
  if (split) AETHER_CUDA_TRY(cudaStreamWaitEvent(sin, ec, 0), "csa_decode_paged_host: order input copy");
  AETHER_CUDA_TRY(cudaMemcpyAsync(dev_in, host_in, in_bytes, cudaMemcpyHostToDevice, sin),
                  "csa_decode_paged_host: input copy");
  if (flags) {
    if (int rc = write_seq(sin, slot_flags, seq, "input flag")) return rc;
  } else if (split) {
    AETHER_CUDA_TRY(cudaEventRecord(eh, sin), "csa_decode_paged_host: record input copy");
    AETHER_CUDA_TRY(cudaStreamWaitEvent(st, eh, 0), "csa_decode_paged_host: wait input copy");
    AETHER_CUDA_TRY(cudaStreamWaitEvent(st, ed, 0), "csa_decode_paged_host: wait output slot");
  }
  const int rc = csa_decode_cta(q, index_q, index_w, sink, window, window_len, idx_pages, kv_pages, page_table,
                                table_stride, num_pages, nblocks, max_nblocks, diag_idx, diag_kv, B, H, W, bits,
                                top_k, softmax_scale, out, sel_out, nullptr, 0, workspace, err, pdl, stream, nullptr,
                                nullptr, 0, flags ? slot_flags : nullptr, seq);
  if (rc) return rc;
  if (split) {
    AETHER_CUDA_TRY(cudaEventRecord(ec, st), "csa_decode_paged_host: record decode");
    AETHER_CUDA_TRY(cudaStreamWaitEvent(sout, ec, 0), "csa_decode_paged_host: wait decode");
  }
  AETHER_CUDA_TRY(cudaMemcpyAsync(host_out, dev_out, out_bytes, cudaMemcpyDeviceToHost, sout),
                  "csa_decode_paged_host: output copy");
  if (flags) {
    if (int rc2 = write_seq(sout, slot_flags + 1, seq, "output flag")) return rc2;
  }
  if (split) AETHER_CUDA_TRY(cudaEventRecord(ed, sout), "csa_decode_paged_host: record output copy");
  return 0;
}

// A prepared host-buffer decode: the staging slots, copy streams, events,
// cache and launch shape bound once, so a step passes only what changes
// between steps (its host buffers, the layer's page table, sink and window).
// Steps alternate between the two staging slots.
struct CsaHostPlan {
  uint8_t* dev_in[2];
  uint8_t* dev_out[2];
  uint32_t* flags[2];
  uint32_t seq[2];
  cudaEvent_t ev[2][3];
  cudaEvent_t fence;
  cudaStream_t h2d, d2h;
  size_t in_bytes, out_bytes, in_off[5], out_off[2];
  const uint8_t* idx_pages;
  const uint8_t* kv_pages;
  int table_stride, num_pages;  // table_stride: the widest page table a step may pass
  const float* diag_idx;
  const float* diag_kv;
  int B, H, W, bits, top_k, pdl, next;
  uint32_t* workspace;
  int* err;
};

static void destroy_host_plan(CsaHostPlan* p) {
  if (!p) return;
  if (p->h2d) cudaStreamSynchronize(p->h2d);
  if (p->d2h) cudaStreamSynchronize(p->d2h);
  for (auto& slot : p->ev)
    for (cudaEvent_t e : slot)
      if (e) cudaEventDestroy(e);
  if (p->fence) cudaEventDestroy(p->fence);
  if (p->h2d) cudaStreamDestroy(p->h2d);
  if (p->d2h) cudaStreamDestroy(p->d2h);
  delete p;
}

int aether_csa_decode_host_plan_create(void* dev_in0, void* dev_in1, size_t in_bytes, const size_t* in_offsets,
                                       void* dev_out0, void* dev_out1, size_t out_bytes, const size_t* out_offsets,
                                       uint32_t* slot_flags, const uint8_t* idx_pages, const uint8_t* kv_pages,
                                       int table_stride, int num_pages, int max_nblocks, const float* diag_idx,
                                       const float* diag_kv, int B, int H, int W, int bits, int top_k,
                                       uint32_t* workspace, int* err, int pdl, void** plan_out) {
  AETHER_REQUIRE(plan_out, "csa_decode_host_plan_create: null plan_out");
  *plan_out = nullptr;
  AETHER_REQUIRE(dev_in0 && dev_in1 && dev_out0 && dev_out1 && slot_flags && in_offsets && out_offsets,
                 "csa_decode_host_plan_create: null staging buffer");
  AETHER_REQUIRE(idx_pages && kv_pages && diag_idx && diag_kv && workspace,
                 "csa_decode_host_plan_create: null cache, diagonal or workspace");
  AETHER_REQUIRE(table_stride > 0 && max_nblocks == table_stride * kPage,
                 "csa_decode_host_plan_create: max_nblocks must be table_stride * %d", kPage);
  for (int i = 0; i < 5; ++i)
    AETHER_REQUIRE(in_offsets[i] < in_bytes && in_offsets[i] % 16 == 0,
                   "csa_decode_host_plan_create: input field %d offset out of range or unaligned", i);
  for (int i = 0; i < 2; ++i)
    AETHER_REQUIRE(out_offsets[i] < out_bytes && out_offsets[i] % 16 == 0,
                   "csa_decode_host_plan_create: output field %d offset out of range or unaligned", i);
  CsaHostPlan* p = new CsaHostPlan{};
  p->dev_in[0] = static_cast<uint8_t*>(dev_in0);
  p->dev_in[1] = static_cast<uint8_t*>(dev_in1);
  p->dev_out[0] = static_cast<uint8_t*>(dev_out0);
  p->dev_out[1] = static_cast<uint8_t*>(dev_out1);
  p->flags[0] = slot_flags;
  p->flags[1] = slot_flags + 2;
  p->in_bytes = in_bytes;
  p->out_bytes = out_bytes;
  for (int i = 0; i < 5; ++i) p->in_off[i] = in_offsets[i];
  for (int i = 0; i < 2; ++i) p->out_off[i] = out_offsets[i];
  p->idx_pages = idx_pages;
  p->kv_pages = kv_pages;
  p->table_stride = table_stride;
  p->num_pages = num_pages;
  p->diag_idx = diag_idx;
  p->diag_kv = diag_kv;
  p->B = B;
  p->H = H;
  p->W = W;
  p->bits = bits;
  p->top_k = top_k;
  p->workspace = workspace;
  p->err = err;
  p->pdl = pdl;
  cudaError_t e = cudaStreamCreateWithFlags(&p->h2d, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p->d2h, cudaStreamNonBlocking);
  for (auto& slot : p->ev)
    for (cudaEvent_t& ev : slot)
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->fence, cudaEventDisableTiming);
  if (e != cudaSuccess) {
    destroy_host_plan(p);
    AETHER_CUDA_TRY(e, "csa_decode_host_plan_create: streams and events");
  }
  *plan_out = p;
  return 0;
}

// One step of a prepared host-buffer decode (aether_csa_decode_paged_host
// on the plan's next staging slot).  After a failed step the plan's slot
// sequence is out of step with its flags: destroy the plan.
int aether_csa_decode_host_plan_step(void* plan, const void* host_in, void* host_out, const int32_t* page_table,
                                     int table_stride, const float* sink, const void* window, float softmax_scale,
                                     void* stream) {
  CsaHostPlan* p = static_cast<CsaHostPlan*>(plan);
  AETHER_REQUIRE(p && host_in && host_out && page_table && sink && window,
                 "csa_decode_host_plan_step: null argument");
  AETHER_REQUIRE(table_stride > 0 && table_stride <= p->table_stride,
                 "csa_decode_host_plan_step: page-table width %d outside (0, %d]", table_stride, p->table_stride);
  const int s = p->next;
  p->next ^= 1;
  const uint32_t seq = ++p->seq[s];
  uint8_t* in = p->dev_in[s];
  uint8_t* out = p->dev_out[s];
  return aether_csa_decode_paged_host(
      host_in, in, p->in_bytes, host_out, out, p->out_bytes, in + p->in_off[0],
      reinterpret_cast<const float*>(in + p->in_off[1]), reinterpret_cast<const float*>(in + p->in_off[2]), sink,
      window, reinterpret_cast<const int32_t*>(in + p->in_off[3]), p->idx_pages, p->kv_pages, page_table,
      table_stride, p->num_pages, reinterpret_cast<const int32_t*>(in + p->in_off[4]), table_stride * 64,
      p->diag_idx, p->diag_kv, p->B, p->H, p->W, p->bits, p->top_k, softmax_scale, out + p->out_off[0],
      reinterpret_cast<int32_t*>(out + p->out_off[1]), p->workspace, p->err, p->pdl, stream, p->h2d, p->d2h,
      p->ev[s][0], p->ev[s][1], p->ev[s][2], p->flags[s], seq);
}

// Orders the plan's copy streams against `stream`: with wait_for_copies 0,
// later copies start after the work enqueued on `stream` so far; with 1,
// later work on `stream` starts after every copy enqueued by the plan so far.
int aether_csa_decode_host_plan_fence(void* plan, void* stream, int wait_for_copies) {
  CsaHostPlan* p = static_cast<CsaHostPlan*>(plan);
  AETHER_REQUIRE(p, "csa_decode_host_plan_fence: null plan");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (wait_for_copies) {
    AETHER_CUDA_TRY(cudaEventRecord(p->fence, p->h2d), "csa_decode_host_plan_fence: record");
    AETHER_CUDA_TRY(cudaStreamWaitEvent(st, p->fence, 0), "csa_decode_host_plan_fence: wait");
    AETHER_CUDA_TRY(cudaEventRecord(p->fence, p->d2h), "csa_decode_host_plan_fence: record");
    AETHER_CUDA_TRY(cudaStreamWaitEvent(st, p->fence, 0), "csa_decode_host_plan_fence: wait");
  } else {
    AETHER_CUDA_TRY(cudaEventRecord(p->fence, st), "csa_decode_host_plan_fence: record");
    AETHER_CUDA_TRY(cudaStreamWaitEvent(p->h2d, p->fence, 0), "csa_decode_host_plan_fence: wait");
    AETHER_CUDA_TRY(cudaStreamWaitEvent(p->d2h, p->fence, 0), "csa_decode_host_plan_fence: wait");
  }
  return 0;
}

// Waits for the plan's copies and frees its streams and events (not the
// caller's buffers).
void aether_csa_decode_host_plan_destroy(void* plan) { destroy_host_plan(static_cast<CsaHostPlan*>(plan)); }

int aether_hca_decode_paged(const void* q, const float* sink, const void* window, const int32_t* window_len,
                            const uint8_t* kv_pages, const int32_t* page_table,
                            int table_stride, int num_pages, const int32_t* nblocks, int max_nblocks,
                            const float* diag_kv, int B, int H, int W, int bits, float softmax_scale, void* out,
                            int* err, int cluster, int pdl, void* stream) {
  if (cluster <= 0)
    return hca_decode_cta(q, sink, window, window_len, kv_pages, page_table, table_stride, num_pages, nblocks,
                          max_nblocks, diag_kv, B, H, W, bits, softmax_scale, out, err, pdl, stream);
  return csa_common(true, q, nullptr, nullptr, sink, window, window_len, nullptr, kv_pages,
                    page_table, table_stride, num_pages, nblocks, max_nblocks, nullptr, diag_kv, B, H, W, bits, 0,
                    softmax_scale, out, nullptr, err, cluster, stream);
}

// Same as aether_csa_decode_paged, and additionally writes every visible
// block's index score to score_out[b * score_stride + block] (fp32).
int aether_csa_decode_paged_scores(const void* q, const float* index_q, const float* index_w, const float* sink,
                                   const void* window, const int32_t* window_len, const uint8_t* idx_pages, const uint8_t* kv_pages,
                                   const int32_t* page_table, int table_stride, int num_pages,
                                   const int32_t* nblocks, int max_nblocks, const float* diag_idx,
                                   const float* diag_kv, int B, int H, int W, int bits, int top_k,
                                   float softmax_scale, void* out, int32_t* sel_out, float* score_out,
                                   int score_stride, uint32_t* workspace, int* err, int cluster, int pdl,
                                   void* stream) {
  AETHER_REQUIRE(index_q && index_w && idx_pages && diag_idx, "csa_decode_paged: null index input");
  AETHER_REQUIRE(score_out && score_stride >= max_nblocks, "score_out must hold max_nblocks per row");
  if (cluster <= 1)
    return csa_decode_cta(q, index_q, index_w, sink, window, window_len, idx_pages, kv_pages, page_table,
                          table_stride, num_pages, nblocks, max_nblocks, diag_idx, diag_kv, B, H, W, bits, top_k,
                          softmax_scale, out, sel_out, score_out, score_stride, workspace, err, pdl, stream);
  return csa_common(false, q, index_q, index_w, sink, window, window_len, idx_pages, kv_pages,
                    page_table, table_stride, num_pages, nblocks, max_nblocks, diag_idx, diag_kv, B, H, W, bits,
                    top_k, softmax_scale, out, sel_out, err, cluster, stream, score_out, score_stride);
}

}  // extern "C"
