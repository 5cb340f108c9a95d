// Fused CSA decode, one CTA per query (sm_100a).
//
// Semantics (reference itz-sayak/deepseek-v4-codebase):
//   indexer   score[s] = sum_h softplus(w_h) * relu(q_h . k_s)   (aether_2b/modeling.py:609-611)
//   top-k     exact top min(top_k, nb), order (score desc, index asc)  (modeling.py:615)
//   attention softmax over [selected compressed ; sliding window] with a
//             per-head sink logit, K == V (aether_pipeline/serving.py:99-130,
//             aether_2b/serving.py:597-625)
//   dequant   decode(c) = diag * WHT(c * s)  (aether_2b/turbo_quant.py:168-211)
//
// The cache stores y = WHT(diag * x) codes; since the normalised WHT is
// symmetric and orthogonal, q . decode(c) = s * (WHT(diag * q) . c): queries
// are rotated once, the codes are used directly, the weighted sum of the
// compressed values stays in the rotated domain and is rotated back once per
// head at the end.  The bf16 window is not rotated and accumulates apart.
//
// Organisation of one CTA (512 threads, 16 warps):
//   producer  warp 15 streams the query's index pages (one TMA bulk copy per
//             page: 64 code rows followed by 64 fp32 scales) through a
//             multi-stage shared-memory ring, gated by full/empty mbarriers.
//             It reads only the page table and the cache, so with
//             programmatic dependent launch it starts before the previous
//             kernel in the stream has finished.
//   scoring   warps 0-14 score 16-key tiles with exact s8 tensor-core dots:
//             the rotated index query is quantised to 24-bit fixed point and
//             split into three signed 8-bit limbs; 4-bit codes enter as
//             (v + 8) and the offset is removed by the accumulator's initial
//             value.  Each score also increments a 4096-bin histogram of its
//             top bits.
//   select    the histogram gives the bin holding rank k; the few keys in that
//             bin are ranked exactly (or, if many, refined by two more radix
//             levels) giving the threshold key T and how many keys equal to T
//             to take; one ordered compaction writes the selected block ids
//             in ascending order (lowest index wins ties).
//   attention the selected rows are gathered with cp.async through the page
//             table staged in shared memory; QK^T and PV run on mma.sync.f16
//             with codes converted to fp16 in registers; the window, fetched
//             into padded rows with cp.async, uses bf16 ldmatrix operands.
//             One warp per head adds the inverse-rotated compressed part to
//             the window part, normalises with the sink and stores bf16.
#include "capi_util.cuh"
#include "common.cuh"

namespace aether {

constexpr int kQThreads = 512;
constexpr int kQWarps = kQThreads / 32;
constexpr int kConsumers = kQWarps - 1;  // warp 15 is the producer
constexpr int kMaxKeys = 8192;           // visible blocks per query (32K tokens at compression 4)
constexpr int kMaxTopK = 256;
constexpr int kWinMax = 128;
constexpr int kWRow = kHeadDim * 2 + 16;  // padded bf16 window row (bytes)
constexpr int kL1Bins = 4096;             // histogram of key >> 19
constexpr int kRankMax = 512;             // boundary-bin size ranked exactly

template <int BITS>
struct QCfg {
  static constexpr int RB_IDX = kIdxDim * BITS / 8;
  static constexpr int RB_KV = kHeadDim * BITS / 8;
  static constexpr int PB_IDX = page_bytes(RB_IDX);
  static constexpr int PB_KV = page_bytes(RB_KV);
  static constexpr int RAWS = RB_KV + 16;          // padded stride of gathered code rows
  static constexpr int CH = BITS == 4 ? 8 : 4;     // pages per ring stage
  static constexpr int STAGES = BITS == 4 ? 6 : 7;
  static constexpr int STAGE_BYTES = CH * PB_IDX;
  static constexpr int RING = STAGES * STAGE_BYTES;
  // attention buffers alias the ring once scoring is over
  static constexpr int LST = kMaxTopK + kWinMax;             // logit row stride (floats)
  static constexpr int PST = kMaxTopK + kWinMax + 8;         // P row stride (halves)
  static constexpr int A_RAW = 0;                            // [256][RAWS]
  static constexpr int A_KS = A_RAW + kMaxTopK * RAWS;       // fp32 [256]
  static constexpr int A_QR = A_KS + kMaxTopK * 4;           // f16 [16][136] rotated, permuted q
  static constexpr int A_QW = A_QR + 16 * 136 * 2;           // bf16 [16][136] plain q
  static constexpr int A_LOG = A_QW + 16 * 136 * 2;          // fp32 [16][LST]
  static constexpr int A_P = A_LOG + 16 * LST * 4;           // f16 [16][PST]
  static constexpr int A_O = A_P + 16 * PST * 2;             // fp32 [2][16][128]
  static constexpr int A_END = A_O + 2 * 16 * kHeadDim * 4;
  static constexpr int REGION = RING > A_END ? RING : A_END;
  static constexpr int A_CAND = 0;                           // u32 [8192] candidate ids (select phase)
  static_assert(kMaxKeys * 4 <= REGION, "candidate list fits");

  static constexpr int OFF_WIN = REGION;                     // bf16 [128][kWRow]
  static constexpr int OFF_SCORES = OFF_WIN + kWinMax * kWRow;
  static constexpr int OFF_HIST = OFF_SCORES + kMaxKeys * 4;  // u32 [4096]
  static constexpr int OFF_PT = OFF_HIST + kL1Bins * 4;       // i32 [128]
  static constexpr int OFF_SEL = OFF_PT + (kMaxKeys / kPage) * 4;  // i32 [256]
  static constexpr int OFF_SCAN = OFF_SEL + kMaxTopK * 4;     // u32 [64]
  static constexpr int OFF_LIMB = OFF_SCAN + 64 * 4;          // s8 [4 heads][3 limbs][64]
  static constexpr int OFF_MISC = OFF_LIMB + kIdxHeads * 3 * kIdxDim;
  static constexpr int MISC_BYTES = 512;
  static constexpr int OFF_BAR = OFF_MISC + MISC_BYTES;       // full[STAGES], empty[STAGES]
  static constexpr int SMEM = OFF_BAR + 8 * 2 * STAGES;
};

struct QParams {
  const __nv_bfloat16* q;
  const float* index_q;
  const float* index_w;
  const float* sink;
  const __nv_bfloat16* window;
  const int32_t* window_len;
  const uint8_t* idx_pages;
  const uint8_t* kv_pages;
  const int32_t* page_table;
  const int32_t* nblocks;
  const float* diag_idx;
  const float* diag_kv;
  __nv_bfloat16* out;
  int32_t* sel_out;
  float* score_out;
  int score_stride;
  int* err;
  int table_stride, num_pages, H, W, top_k;
  float softmax_scale;
};

struct QMisc {
  float alpha[kIdxHeads];
  float qscale[kIdxHeads];
  int lsum[kIdxHeads][3];  // sum over dims of each limb (4-bit offset correction)
  int bin;
  uint32_t above;
  uint32_t cnt;
  uint32_t ncand;
  uint32_t thr;
  uint32_t take_eq;
  float m_h[kMaxHeads];
  float l_h[kMaxHeads];
};

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// Block-wide inclusive scan of one u32 per thread (512 threads); uses wtot[0..31].
__device__ __forceinline__ uint32_t block_scan_incl(uint32_t v, uint32_t* wtot, int lane, int warp) {
  uint32_t inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t u = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += u;
  }
  if (lane == 31) wtot[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < kQWarps ? wtot[lane] : 0u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t u = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += u;
    }
    if (lane < kQWarps) wtot[16 + lane] = w;
  }
  __syncthreads();
  return (warp ? wtot[16 + warp - 1] : 0u) + inc;
}

// Bin holding the R-th largest element of a histogram scanned from the top
// bin down; writes bin, count above it and count in it to misc.
__device__ __forceinline__ void find_bin(const uint32_t* hist, int nbins, uint32_t R, uint32_t* wtot, QMisc* misc,
                                         int tid, int lane, int warp) {
  const int per = nbins / kQThreads;
  uint32_t s = 0;
  for (int k = 0; k < per; ++k) s += hist[nbins - 1 - (tid * per + k)];
  const uint32_t inc = block_scan_incl(s, wtot, lane, warp);
  const uint32_t exc = inc - s;
  if (exc < R && inc >= R) {
    uint32_t cum = exc;
    for (int k = 0; k < per; ++k) {
      const int bin = nbins - 1 - (tid * per + k);
      const uint32_t v = hist[bin];
      if (cum + v >= R) {
        misc->bin = bin;
        misc->above = cum;
        misc->cnt = v;
        break;
      }
      cum += v;
    }
  }
  __syncthreads();
}

// warp-aggregated histogram increment (lanes with bin < 0 do not count)
__device__ __forceinline__ void hist_add(uint32_t* hist, int bin, int lane) {
  const uint32_t key = bin >= 0 ? static_cast<uint32_t>(bin) : 0xFFFFFFFFu;
  const uint32_t peers = __match_any_sync(0xffffffffu, key);
  if (bin >= 0 && (__ffs(peers) - 1) == lane) atomicAdd(&hist[bin], __popc(peers));
}

// nibble pair of one byte -> half2(lo, hi), exact signed values
__device__ __forceinline__ uint32_t nib_byte_to_h2(uint32_t byte) {
  uint32_t y = (byte & 0xFu) | ((byte & 0xF0u) << 12);
  y = (y ^ 0x00080008u) | 0x64006400u;
  __half2 h = *reinterpret_cast<__half2*>(&y);
  h = __hsub2(h, __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408)));  // 1032
  return *reinterpret_cast<uint32_t*>(&h);
}
// two int8 codes (low 16 bits of w) -> half2
__device__ __forceinline__ uint32_t s8pair_to_h2(uint32_t w) {
  uint32_t y = __byte_perm(w ^ 0x8080u, 0x64646464u, 0x5140);  // [b0^80, 0x64, b1^80, 0x64]
  __half2 h = *reinterpret_cast<__half2*>(&y);
  h = __hsub2(h, __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480)));  // 1152
  return *reinterpret_cast<uint32_t*>(&h);
}
// selected nibble (shift sh) of two bytes -> half2
__device__ __forceinline__ uint32_t two_nib_to_h2(uint32_t b0, uint32_t b1, int sh) {
  uint32_t y = ((b0 >> sh) & 0xFu) | (((b1 >> sh) & 0xFu) << 16);
  y = (y ^ 0x00080008u) | 0x64006400u;
  __half2 h = *reinterpret_cast<__half2*>(&y);
  h = __hsub2(h, __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408)));
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t two_s8_to_h2(uint32_t b0, uint32_t b1) {
  return s8pair_to_h2((b0 & 0xFFu) | ((b1 & 0xFFu) << 8));
}
__device__ __forceinline__ uint32_t bf2_to_h2(uint32_t v) {
  const __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v);
  const float2 f = __bfloat1622float2(b);
  return pack_half2(f.x, f.y);
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// In-warp normalised 128-point WHT of 4 consecutive values per lane (unscaled).
__device__ __forceinline__ void warp_wht128(float (&v)[4], int lane) {
  {
    const float a0 = v[0] + v[1], a1 = v[0] - v[1], a2 = v[2] + v[3], a3 = v[2] - v[3];
    v[0] = a0 + a2;
    v[2] = a0 - a2;
    v[1] = a1 + a3;
    v[3] = a1 - a3;
  }
#pragma unroll
  for (int ld = 1; ld < 32; ld <<= 1) {
    const bool up = (lane & ld) != 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float o = __shfl_xor_sync(0xffffffffu, v[k], ld);
      v[k] = up ? o - v[k] : v[k] + o;
    }
  }
}

template <int BITS>
__global__ void __launch_bounds__(kQThreads, 1) csa_decode_cta_kernel(QParams p) {
  using C = QCfg<BITS>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  pdl_launch_dependents();

  uint8_t* winb = smem + C::OFF_WIN;
  uint32_t* scores = reinterpret_cast<uint32_t*>(smem + C::OFF_SCORES);
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem + C::OFF_HIST);
  int32_t* pt = reinterpret_cast<int32_t*>(smem + C::OFF_PT);
  int32_t* sel = reinterpret_cast<int32_t*>(smem + C::OFF_SEL);
  uint32_t* wtot = reinterpret_cast<uint32_t*>(smem + C::OFF_SCAN);
  int8_t* limb = reinterpret_cast<int8_t*>(smem + C::OFF_LIMB);
  QMisc* misc = reinterpret_cast<QMisc*>(smem + C::OFF_MISC);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* empty = full + C::STAGES;

  // ------------------------------------------------------------ prologue
  int nb = p.nblocks[b];
  if (nb > kMaxKeys || nb > p.table_stride * kPage) {
    if (tid == 0) report_error(p.err, kErrBadShape);
    nb = min(kMaxKeys, p.table_stride * kPage);
  }
  nb = max(nb, 0);
  const int K = min(p.top_k, nb);
  const int npages = (nb + kPage - 1) / kPage;
  const int nchunks = (npages + C::CH - 1) / C::CH;
  const int W = p.W;
  const int wl = max(0, min(p.window_len[b], W));
  const int32_t* ptab = p.page_table + static_cast<long long>(b) * p.table_stride;
  for (int i = tid; i < npages; i += kQThreads) {
    int v = ptab[i];
    if (v < 0 || v >= p.num_pages) {
      report_error(p.err, kErrBadPage);
      v = 0;
    }
    pt[i] = v;
  }
  for (int i = tid; i < kL1Bins; i += kQThreads) hist[i] = 0;
  if (tid == 0) {
    for (int i = 0; i < C::STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kConsumers);
    }
    fence_mbar_init();
  }
  __syncthreads();

  // window rows other than the newest are cache state: prefetch them now
  {
    const int pre = max(wl - 1, 0);
    const __nv_bfloat16* wsrc = p.window + static_cast<long long>(b) * W * kHeadDim;
    for (int i = tid; i < pre * 16; i += kQThreads)
      cp_async16(winb + (i >> 4) * kWRow + (i & 15) * 16, wsrc + (i >> 4) * kHeadDim + (i & 15) * 8);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }

  if (warp == kQWarps - 1) {
    // ---------------------------------------------------------- producer
    for (int c = 0; c < nchunks; ++c) {
      const int stage = c % C::STAGES;
      if (c >= C::STAGES) mbar_wait(&empty[stage], ((c / C::STAGES) - 1) & 1, p.err);
      const int np = min(C::CH, npages - c * C::CH);
      if (lane == 0) mbar_expect_tx(&full[stage], np * C::PB_IDX);
      __syncwarp();
      if (lane < np)
        bulk_g2s(smem + stage * C::STAGE_BYTES + lane * C::PB_IDX,
                 p.idx_pages + static_cast<long long>(pt[c * C::CH + lane]) * C::PB_IDX, C::PB_IDX, &full[stage]);
    }
    pdl_wait();
  } else {
    // everything below may depend on the previous kernel in the stream
    pdl_wait();
    if (warp < kIdxHeads) {
      // rotated index query, 24-bit limbs, alpha_h = softplus(w_h) * scale_h
      const int h = warp;
      const float* src = p.index_q + (static_cast<long long>(b) * kIdxHeads + h) * kIdxDim;
      float v0 = src[lane * 2] * p.diag_idx[lane * 2];
      float v1 = src[lane * 2 + 1] * p.diag_idx[lane * 2 + 1];
      {
        const float a = v0, c2 = v1;
        v0 = a + c2;
        v1 = a - c2;
      }
#pragma unroll
      for (int ld = 1; ld < 32; ld <<= 1) {
        const bool up = (lane & ld) != 0;
        const float o0 = __shfl_xor_sync(0xffffffffu, v0, ld);
        const float o1 = __shfl_xor_sync(0xffffffffu, v1, ld);
        v0 = up ? o0 - v0 : v0 + o0;
        v1 = up ? o1 - v1 : v1 + o1;
      }
      v0 *= 0.125f;
      v1 *= 0.125f;
      const float am = warp_max(fmaxf(fabsf(v0), fabsf(v1)));
      const float s = am > 0.f ? am / 8355000.0f : 1.0f;
      int ls[3] = {0, 0, 0};
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int v = __float2int_rn(__fdiv_rn(k ? v1 : v0, s));
        const int l0 = ((v + 128) & 255) - 128;
        const int w1 = (v - l0) >> 8;
        const int l1 = ((w1 + 128) & 255) - 128;
        const int l2 = (w1 - l1) >> 8;
        const int d = lane * 2 + k;
        limb[(h * 3 + 0) * kIdxDim + d] = static_cast<int8_t>(l0);
        limb[(h * 3 + 1) * kIdxDim + d] = static_cast<int8_t>(l1);
        limb[(h * 3 + 2) * kIdxDim + d] = static_cast<int8_t>(l2);
        ls[0] += l0;
        ls[1] += l1;
        ls[2] += l2;
      }
#pragma unroll
      for (int l = 0; l < 3; ++l) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ls[l] += __shfl_xor_sync(0xffffffffu, ls[l], o);
      }
      if (lane == 0) {
        misc->qscale[h] = s;
        misc->alpha[h] = softplus_f(p.index_w[b * kIdxHeads + h]) * s;
        misc->lsum[h][0] = ls[0];
        misc->lsum[h][1] = ls[1];
        misc->lsum[h][2] = ls[2];
      }
    }
    // consumers only: named barrier 1 over warps 0..14
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");

    // B fragments: column n = g of n-tile 0 is (head g/2, limb g%2), of
    // n-tile 1 (head g/2, limb 2) for even g and zero for odd g.
    uint32_t bq[2][2][2];
    {
      const int hq = g >> 1;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t w0 = 0, w1 = 0;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int d = BITS == 4 ? 16 * t + 8 * j + 2 * e + hh : 16 * t + 8 * j + 4 * hh + e;
            const int lA = limb[(hq * 3 + (g & 1)) * kIdxDim + d];
            const int lB = (g & 1) ? 0 : limb[(hq * 3 + 2) * kIdxDim + d];
            w0 |= (static_cast<uint32_t>(lA) & 0xFFu) << (8 * e);
            w1 |= (static_cast<uint32_t>(lB) & 0xFFu) << (8 * e);
          }
          bq[0][j][hh] = w0;
          bq[1][j][hh] = w1;
        }
    }
    const float alpha_t = misc->alpha[t];
    // 4-bit codes enter the MMA as v + 8; start the accumulators at
    // -8 * sum(limb) so the dot products come out exact.
    const int c0i = BITS == 4 ? -8 * misc->lsum[t][0] : 0;
    const int c1i = BITS == 4 ? -8 * misc->lsum[t][1] : 0;
    const int c2i = BITS == 4 ? -8 * misc->lsum[t][2] : 0;

    // ------------------------------------------------------------ scoring
    for (int c = 0; c < nchunks; ++c) {
      const int stage = c % C::STAGES;
      mbar_wait(&full[stage], (c / C::STAGES) & 1, p.err);
      const uint8_t* stg = smem + stage * C::STAGE_BYTES;
      const int np = min(C::CH, npages - c * C::CH);
      const int tiles = np * (kPage / 16);
      for (int tile = warp; tile < tiles; tile += kConsumers) {
        const uint8_t* page = stg + (tile >> 2) * C::PB_IDX;
        const float* ksc = reinterpret_cast<const float*>(page + kPage * C::RB_IDX);
        const int ra = (tile & 3) * 16 + g, rb = ra + 8;  // slots in the page
        uint32_t a[2][4];
        if (BITS == 4) {
          const uint2 va = *reinterpret_cast<const uint2*>(page + ra * C::RB_IDX + t * 8);
          const uint2 vb = *reinterpret_cast<const uint2*>(page + rb * C::RB_IDX + t * 8);
          a[0][0] = (va.x & 0x0F0F0F0Fu) ^ 0x08080808u;
          a[0][2] = ((va.x >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
          a[0][1] = (vb.x & 0x0F0F0F0Fu) ^ 0x08080808u;
          a[0][3] = ((vb.x >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
          a[1][0] = (va.y & 0x0F0F0F0Fu) ^ 0x08080808u;
          a[1][2] = ((va.y >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
          a[1][1] = (vb.y & 0x0F0F0F0Fu) ^ 0x08080808u;
          a[1][3] = ((vb.y >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
        } else {
          const uint4 va = *reinterpret_cast<const uint4*>(page + ra * C::RB_IDX + t * 16);
          const uint4 vb = *reinterpret_cast<const uint4*>(page + rb * C::RB_IDX + t * 16);
          a[0][0] = va.x; a[0][1] = vb.x; a[0][2] = va.y; a[0][3] = vb.y;
          a[1][0] = va.z; a[1][1] = vb.z; a[1][2] = va.w; a[1][3] = vb.w;
        }
        int acc0[4] = {c0i, c1i, c0i, c1i}, acc1[4] = {c2i, 0, c2i, 0};
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          mma_s8(acc0, a[j][0], a[j][1], a[j][2], a[j][3], bq[0][j][0], bq[0][j][1]);
          mma_s8(acc1, a[j][0], a[j][1], a[j][2], a[j][3], bq[1][j][0], bq[1][j][1]);
        }
        // thread t holds head t: limbs (acc0[0], acc0[1], acc1[0]) for row a,
        // (acc0[2], acc0[3], acc1[2]) for row b
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
        int bin = -1;
        if (t < 2) {
          const int slot = t == 0 ? ra : rb;
          const int key = (c * C::CH + (tile >> 2)) * kPage + slot;
          if (key < nb) {
            const float s = __fadd_rn(__fmul_rn(t == 0 ? sA : sB, ksc[slot]), 0.0f);
            const uint32_t kv = __float_as_uint(s) + 1u;
            scores[key] = kv;
            bin = static_cast<int>(kv >> 19);
          }
        }
        hist_add(hist, bin, lane);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
    }
  }
  __syncthreads();
  if (p.score_out) {
    float* so = p.score_out + static_cast<long long>(b) * p.score_stride;
    for (int i = tid; i < nb; i += kQThreads) so[i] = __uint_as_float(scores[i] - 1u);
  }

  // ------------------------------------------------------------- select
  // Result: every key > thr is taken, and the take_eq lowest-index keys == thr.
  if (tid == 0) {
    misc->thr = 0;
    misc->take_eq = 0xFFFFFFFFu;
    misc->ncand = 0;
  }
  __syncthreads();
  if (nb > K) {
    uint32_t R = static_cast<uint32_t>(K);
    find_bin(hist, kL1Bins, R, wtot, misc, tid, lane, warp);
    const uint32_t b1 = misc->bin;
    R -= misc->above;
    if (misc->cnt == R) {
      if (tid == 0) misc->thr = b1 << 19;  // lowest key of bin b1: all of the bin is taken
    } else {
      uint32_t* cand = reinterpret_cast<uint32_t*>(smem + C::A_CAND);
      for (int base = 0; base < nb; base += kQThreads) {
        const int i = base + tid;
        const bool m = i < nb && (scores[i] >> 19) == b1;
        const uint32_t bal = __ballot_sync(0xffffffffu, m);
        uint32_t off = 0;
        if (lane == 0 && bal) off = atomicAdd(&misc->ncand, __popc(bal));
        off = __shfl_sync(0xffffffffu, off, 0);
        if (m) cand[off + __popc(bal & ((1u << lane) - 1))] = static_cast<uint32_t>(i);
      }
      __syncthreads();
      const uint32_t nc = misc->ncand;
      if (nc <= kRankMax) {
        // exact rank of each candidate: (key desc, index asc)
        if (tid < static_cast<int>(nc)) {
          const uint32_t ci = cand[tid], ki = scores[ci];
          uint32_t rank = 0;
          for (uint32_t j = 0; j < nc; ++j) {
            const uint32_t cj = cand[j], kj = scores[cj];
            rank += (kj > ki) || (kj == ki && cj < ci);
          }
          if (rank == R - 1) {
            uint32_t gt = 0;
            for (uint32_t j = 0; j < nc; ++j) gt += scores[cand[j]] > ki;
            misc->thr = ki;
            misc->take_eq = R - gt;
          }
        }
      } else {
        // many keys in the bin (heavy ties): two more radix levels
        for (int i = tid; i < 2048; i += kQThreads) hist[i] = 0;
        __syncthreads();
        for (uint32_t i = tid; i < nc; i += kQThreads) atomicAdd(&hist[(scores[cand[i]] >> 8) & 2047u], 1u);
        __syncthreads();
        find_bin(hist, 2048, R, wtot, misc, tid, lane, warp);
        const uint32_t b2 = misc->bin;
        R -= misc->above;
        for (int i = tid; i < 2048; i += kQThreads) hist[i] = 0;
        __syncthreads();
        for (uint32_t i = tid; i < nc; i += kQThreads) {
          const uint32_t key = scores[cand[i]];
          if (((key >> 8) & 2047u) == b2) atomicAdd(&hist[key & 255u], 1u);
        }
        __syncthreads();
        find_bin(hist, kQThreads, R, wtot, misc, tid, lane, warp);  // 256 used bins of 512
        R -= misc->above;
        if (tid == 0) {
          misc->thr = (b1 << 19) | (b2 << 8) | static_cast<uint32_t>(misc->bin);
          misc->take_eq = R;
        }
      }
    }
  }
  __syncthreads();
  // ordered compaction: warp w owns keys [512w, 512w + 512)
  {
    const uint32_t thr = misc->thr, take_eq = misc->take_eq;
    const int base = warp * 512;
    uint32_t cs = 0, ce = 0;
    for (int r = 0; r < 16; ++r) {
      const int i = base + r * 32 + lane;
      const uint32_t key = i < nb ? scores[i] : 0u;
      cs += __popc(__ballot_sync(0xffffffffu, i < nb && key > thr));
      ce += __popc(__ballot_sync(0xffffffffu, i < nb && key == thr));
    }
    if (lane == 0) {
      wtot[32 + warp] = cs;
      wtot[48 + warp] = ce;
    }
    __syncthreads();
    uint32_t sb = 0, eb = 0;
    for (int w = 0; w < warp; ++w) {
      sb += wtot[32 + w];
      eb += wtot[48 + w];
    }
    const uint32_t lt = (1u << lane) - 1;
    for (int r = 0; r < 16; ++r) {
      const int i = base + r * 32 + lane;
      const uint32_t key = i < nb ? scores[i] : 0u;
      const bool st = i < nb && key > thr, eq = i < nb && key == thr;
      const uint32_t bs = __ballot_sync(0xffffffffu, st), be = __ballot_sync(0xffffffffu, eq);
      const uint32_t mys = sb + __popc(bs & lt), mye = eb + __popc(be & lt);
      if (st) sel[mys + min(mye, take_eq)] = i;
      if (eq && mye < take_eq) sel[mys + mye] = i;
      sb += __popc(bs);
      eb += __popc(be);
    }
  }
  __syncthreads();
  if (p.sel_out) {
    int32_t* so = p.sel_out + static_cast<long long>(b) * p.top_k;
    for (int i = tid; i < p.top_k; i += kQThreads) so[i] = i < K ? sel[i] : -1;
  }

  // --------------------------------------------------------- attention
  uint8_t* raw = smem + C::A_RAW;
  float* ks = reinterpret_cast<float*>(smem + C::A_KS);
  __half* Qr = reinterpret_cast<__half*>(smem + C::A_QR);
  __nv_bfloat16* Qw = reinterpret_cast<__nv_bfloat16*>(smem + C::A_QW);
  float* logit = reinterpret_cast<float*>(smem + C::A_LOG);
  __half* P = reinterpret_cast<__half*>(smem + C::A_P);
  float* Obuf = reinterpret_cast<float*>(smem + C::A_O);
  const int ntc = (K + 15) / 16, ntw = (wl + 15) / 16;
  {
    constexpr int CPR = C::RB_KV / 16;
    for (int i = tid; i < ntc * 16 * CPR; i += kQThreads) {
      const int row = i / CPR, ch = i % CPR;
      if (row < K) {
        const int blk = sel[row];
        const uint8_t* pg = p.kv_pages + static_cast<long long>(pt[blk >> 6]) * C::PB_KV;
        cp_async16(raw + row * C::RAWS + ch * 16, pg + (blk & 63) * C::RB_KV + ch * 16);
        if (ch == 0) cp_async4(ks + row, pg + kPage * C::RB_KV + (blk & 63) * 4);
      } else {
        *reinterpret_cast<uint4*>(raw + row * C::RAWS + ch * 16) = make_uint4(0, 0, 0, 0);
        if (ch == 0) ks[row] = 0.f;
      }
    }
    // newest window row (written by the previous step)
    if (wl > 0 && tid < 16)
      cp_async16(winb + (wl - 1) * kWRow + tid * 16,
                 p.window + (static_cast<long long>(b) * W + wl - 1) * kHeadDim + tid * 8);
  }
  // queries: plain bf16 rows for the window, rotated fp16 rows permuted to
  // the QK operand layout for the codes
  {
    const int h = warp;  // 16 warps, 16 padded heads
    float v[4];
    if (h < p.H) {
      const uint2 r4 = *reinterpret_cast<const uint2*>(p.q + (static_cast<long long>(b) * p.H + h) * kHeadDim + lane * 4);
      *reinterpret_cast<uint2*>(Qw + h * 136 + lane * 4) = r4;
      const __nv_bfloat162* bb = reinterpret_cast<const __nv_bfloat162*>(&r4);
      const float2 f0 = __bfloat1622float2(bb[0]), f1 = __bfloat1622float2(bb[1]);
      v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
    } else {
      *reinterpret_cast<uint2*>(Qw + h * 136 + lane * 4) = make_uint2(0, 0);
      v[0] = v[1] = v[2] = v[3] = 0.f;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] *= p.diag_kv[lane * 4 + k];
    warp_wht128(v, lane);
    // logical k index c of k-step j reads physical dim 32*(c%8/2) + 4j + 2*(c/8) + c%2
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int d = lane * 4 + k;
      const int tq = d >> 5, rem = d & 31, j = rem >> 2, hi = (rem >> 1) & 1, e = rem & 1;
      Qr[h * 136 + j * 16 + hi * 8 + tq * 2 + e] = __float2half_rn(v[k] * 0.0883883461356163f);
    }
  }
  // zero window rows past wl up to the tile edge
  for (int i = tid; i < (ntw * 16 - wl) * 16; i += kQThreads)
    *reinterpret_cast<uint4*>(winb + (wl + (i >> 4)) * kWRow + (i & 15) * 16) = make_uint4(0, 0, 0, 0);
  cp_async_commit_wait_all();
  __syncthreads();

  // ---- S = Q K^T, one 16-source tile per warp iteration
  {
    uint32_t aq[8][4];
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
      ldsm_x4(aq[kk][0], aq[kk][1], aq[kk][2], aq[kk][3], Qr + (lane & 15) * 136 + kk * 16 + (lane >> 4) * 8);
    for (int tile = warp; tile < ntc + ntw; tile += kQWarps) {
      const bool comp = tile < ntc;
      float acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
      if (comp) {
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const uint8_t* row = raw + (tile * 16 + nt * 8 + g) * C::RAWS;
          if (BITS == 4) {
            const uint4 cv = *reinterpret_cast<const uint4*>(row + t * 16);
            const uint32_t w[4] = {cv.x, cv.y, cv.z, cv.w};
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const uint32_t wd = w[kk >> 1];
              const int sh = (kk & 1) * 16;
              mma_f16(acc[nt], aq[kk], nib_byte_to_h2((wd >> sh) & 0xFFu), nib_byte_to_h2((wd >> (sh + 8)) & 0xFFu));
            }
          } else {
            const uint4 c0 = *reinterpret_cast<const uint4*>(row + t * 32);
            const uint4 c1 = *reinterpret_cast<const uint4*>(row + t * 32 + 16);
            const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) mma_f16(acc[nt], aq[kk], s8pair_to_h2(w[kk] & 0xFFFFu), s8pair_to_h2(w[kk] >> 16));
          }
        }
      } else {
        const uint8_t* wt = winb + (tile - ntc) * 16 * kWRow;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          uint32_t a[4];
          ldsm_x4(a[0], a[1], a[2], a[3], Qw + (lane & 15) * 136 + kk * 16 + (lane >> 4) * 8);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(b0, b1, b2, b3, wt + ((lane & 7) + ((lane >> 4) << 3)) * kWRow + (kk * 16 + ((lane >> 3) & 1) * 8) * 2);
          mma_bf16(acc[0], a, b0, b1);
          mma_bf16(acc[1], a, b2, b3);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int h = g + (e >> 1) * 8;
          const int src = tile * 16 + nt * 8 + 2 * t + (e & 1);
          float z;
          if (comp) z = src < K ? acc[nt][e] * ks[src] * p.softmax_scale : -INFINITY;
          else z = (src - ntc * 16) < wl ? acc[nt][e] * p.softmax_scale : -INFINITY;
          logit[h * C::LST + src] = z;
        }
    }
  }
  __syncthreads();
  // ---- softmax statistics, one warp per head
  const int ncols = (ntc + ntw) * 16, ncc = ntc * 16;
  {
    const int h = warp;
    float m = -INFINITY;
    for (int c = lane; c < ncols; c += 32) m = fmaxf(m, logit[h * C::LST + c]);
    m = warp_max(m);
    const float mu = m == -INFINITY ? 0.f : m;
    float l = 0.f;
    for (int c = lane; c < ncols; c += 32) {
      const float e = __expf(logit[h * C::LST + c] - mu);
      l += e;
      const float w = c < ncc ? (c < K ? e * ks[c] : 0.f) : e;
      P[h * C::PST + c] = __float2half_rn(h < p.H ? w : 0.f);
    }
    l = warp_sum(l);
    if (lane == 0) {
      misc->m_h[h] = m;
      misc->l_h[h] = l;
    }
  }
  __syncthreads();
  // ---- O = P V; warp w owns output dims [8w, 8w+8)
  {
    float orot[4] = {0, 0, 0, 0}, owin[4] = {0, 0, 0, 0};
    const int d = warp * 8 + g;
    for (int kt = 0; kt < ntc; ++kt) {
      uint32_t a[4];
      ldsm_x4(a[0], a[1], a[2], a[3], P + (lane & 15) * C::PST + kt * 16 + (lane >> 4) * 8);
      const uint8_t* r0 = raw + (kt * 16 + 2 * t) * C::RAWS;
      uint32_t b0, b1;
      if (BITS == 4) {
        const int sh = (d & 1) * 4, col = d >> 1;
        b0 = two_nib_to_h2(r0[col], r0[C::RAWS + col], sh);
        b1 = two_nib_to_h2(r0[8 * C::RAWS + col], r0[9 * C::RAWS + col], sh);
      } else {
        b0 = two_s8_to_h2(r0[d], r0[C::RAWS + d]);
        b1 = two_s8_to_h2(r0[8 * C::RAWS + d], r0[9 * C::RAWS + d]);
      }
      mma_f16(orot, a, b0, b1);
    }
    for (int kt = ntc; kt < ntc + ntw; ++kt) {
      uint32_t a[4];
      ldsm_x4(a[0], a[1], a[2], a[3], P + (lane & 15) * C::PST + kt * 16 + (lane >> 4) * 8);
      const uint8_t* wt = winb + (kt - ntc) * 16 * kWRow;
      uint32_t b0, b1;
      asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
                   : "=r"(b0), "=r"(b1)
                   : "r"(smem_u32(wt + ((lane & 7) + ((lane >> 3) & 1) * 8) * kWRow + warp * 16)));
      mma_f16(owin, a, bf2_to_h2(b0), bf2_to_h2(b1));
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int h = g + (e >> 1) * 8;
      const int dd = warp * 8 + 2 * t + (e & 1);
      Obuf[h * kHeadDim + dd] = orot[e];
      Obuf[16 * kHeadDim + h * kHeadDim + dd] = owin[e];
    }
  }
  __syncthreads();
  // ---- per head: inverse rotation, sink, normalise, store
  if (warp < p.H) {
    const int h = warp;
    const float m = misc->m_h[h], l = misc->l_h[h];
    const float sk = p.sink[h];
    const float M = fmaxf(m, sk);
    const float a = m == -INFINITY ? 0.f : __expf(m - M);
    const float inv = a / (l * a + __expf(sk - M));
    const float4 o1 = *reinterpret_cast<const float4*>(Obuf + h * kHeadDim + lane * 4);
    const float4 o2 = *reinterpret_cast<const float4*>(Obuf + 16 * kHeadDim + h * kHeadDim + lane * 4);
    float vr[4] = {o1.x, o1.y, o1.z, o1.w};
    const float vw[4] = {o2.x, o2.y, o2.z, o2.w};
    warp_wht128(vr, lane);
    float o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = (vr[k] * 0.0883883461356163f * p.diag_kv[lane * 4 + k] + vw[k]) * inv;
    __nv_bfloat162 o01 = __floats2bfloat162_rn(o[0], o[1]), o23 = __floats2bfloat162_rn(o[2], o[3]);
    *reinterpret_cast<uint2*>(p.out + (static_cast<long long>(b) * p.H + h) * kHeadDim + lane * 4) =
        make_uint2(*reinterpret_cast<uint32_t*>(&o01), *reinterpret_cast<uint32_t*>(&o23));
  }
}

template <int BITS>
static int launch_q1(const QParams& p, int B, bool pdl, cudaStream_t st) {
  using C = QCfg<BITS>;
  auto kern = csa_decode_cta_kernel<BITS>;
  static bool attr = false;
  if (!attr) {
    AETHER_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM),
                    "csa_decode: set shared memory size");
    attr = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(B);
  cfg.blockDim = dim3(kQThreads);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  AETHER_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p), "csa_decode: launch");
  return check_launch("csa_decode");
}

int csa_decode_cta(const void* q, const float* index_q, const float* index_w, const float* sink, const void* window,
                   const int32_t* window_len, const uint8_t* idx_pages, const uint8_t* kv_pages,
                   const int32_t* page_table, int table_stride, int num_pages, const int32_t* nblocks,
                   int max_nblocks, const float* diag_idx, const float* diag_kv, int B, int H, int W, int bits,
                   int top_k, float softmax_scale, void* out, int32_t* sel_out, float* score_out, int score_stride,
                   int* err, int pdl, void* stream) {
  AETHER_REQUIRE(bits == 4 || bits == 8, "bits must be 4 or 8, got %d", bits);
  AETHER_REQUIRE(H >= 1 && H <= kMaxHeads, "num_heads must be in [1, %d], got %d", kMaxHeads, H);
  AETHER_REQUIRE(W >= 0 && W <= kWinMax, "window capacity must be in [0, %d], got %d", kWinMax, W);
  AETHER_REQUIRE(top_k >= 1 && top_k <= kMaxTopK, "top_k must be in [1, %d], got %d", kMaxTopK, top_k);
  AETHER_REQUIRE(max_nblocks <= kMaxKeys, "csa decode: %d visible blocks exceed the per-query limit %d", max_nblocks,
                 kMaxKeys);
  AETHER_REQUIRE(table_stride >= 1 && num_pages >= 1, "page table / pool must be non-empty");
  if (B == 0) return 0;
  QParams p;
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
  p.top_k = top_k;
  p.softmax_scale = softmax_scale;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return bits == 4 ? launch_q1<4>(p, B, pdl != 0, st) : launch_q1<8>(p, B, pdl != 0, st);
}

}  // namespace aether

extern "C" int aether_csa_decode_smem_bytes(int bits) {
  return bits == 4 ? aether::QCfg<4>::SMEM : aether::QCfg<8>::SMEM;
}
