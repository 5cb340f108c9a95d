// Fused CSA decode over a paged TurboQuant KV cache (sm_100a): two kernels
// chained with programmatic dependent launch.
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
// Kernel A (score): a 256-thread CTA per (sequence, run of 16 index pages).
//   Before griddepcontrol.wait it stages its pages (one TMA bulk copy per
//   page: 64 code rows then 64 fp32 scales) in shared memory; after the wait
//   it scores 16-key tiles with exact s8 tensor-core dots (the rotated index
//   query quantised to 24-bit fixed point and split into three signed 8-bit
//   limbs; 4-bit codes enter as v + 8, the offset removed by the
//   accumulator's initial value) and writes one order-preserving u32 key per
//   block to the workspace (L2 resident).
// Kernel B (select + attend): a 512-thread CTA per sequence.  It prefetches
//   the page-table row and the window rows, waits for kernel A, loads the
//   keys into registers (16 per thread, in index order), builds a 4096-bin
//   histogram of their top bits, finds the bin of rank k, ranks the keys of
//   that bin exactly (radix refinement if there are many), and compacts the
//   winners in ascending index order (lowest index wins ties).  The selected
//   rows are gathered with cp.async; QK^T and PV run on mma.sync.f16 with
//   codes converted to fp16 in registers; the window uses bf16 ldmatrix
//   operands.  One warp per head adds the inverse-rotated compressed part to
//   the window part, normalises with the sink and stores bf16.
#include <cooperative_groups.h>
#include <stdlib.h>

#include "aether_b200.h"
#include "capi_util.cuh"
#include "common.cuh"
#include "decode_common.cuh"

namespace cg = cooperative_groups;

namespace aether {


constexpr int kQThreads = 512;
constexpr int kQWarps = kQThreads / 32;
constexpr int kMaxKeys = 8192;           // visible blocks per query (32K tokens at compression 4)
constexpr int kMaxTopK = 256;
constexpr int kWinMax = 128;
constexpr int kWRow = kHeadDim * 2 + 16;  // padded bf16 window row (bytes)
constexpr int kL1Bins = 4096;            // histogram of key >> 19
constexpr int kBoundMax = 512;           // boundary-bin keys ranked directly (more: radix levels)
constexpr int kMaxPagesLocal = 4096;      // page-table entries per sequence on one device (262144 blocks)
constexpr int kMaxBlocks = kMaxPagesLocal * kPage;

template <int BITS, int CS>
struct QCfg {
  static constexpr int RB_KV = kHeadDim * BITS / 8;
  static constexpr int PB_KV = page_bytes(RB_KV);
  static constexpr int RAWS = RB_KV + 16;                    // padded stride of gathered code rows
  static constexpr int KROW = kHeadDim + 8;                  // fp16 operand row stride (halves)
  static constexpr int SL = kMaxTopK / CS;                   // selected rows attended per CTA (max)
  static constexpr int WSL = kWinMax / CS;                   // window rows per CTA (max)
  // logit row stride (floats), = 8 mod 32: the per-head float2 stores of an
  // MMA tile hit distinct banks
  static constexpr int LST = SL + WSL + 8;
  static constexpr int PST = SL + WSL + 8;                   // P row stride (halves)
  static constexpr int HPC = (kMaxHeads + CS - 1) / CS;      // heads finalised per CTA (max)
  static constexpr int SLOT = 4 + 2 * kHeadDim;              // merge slot: m, l, pad, pad, O_rot, O_win
  // select phase (aliases the attention buffers below)
  static constexpr int S_HIST = 0;                           // u32 [4096], then uint2 [kBoundMax]
  static constexpr int S_END = S_HIST + kL1Bins * 4 + kBoundMax * 8;
  // attention phase
  static constexpr int A_KC = 0;                             // f16 [SL][KROW] expanded codes
  static constexpr int A_KS = A_KC + SL * KROW * 2;          // fp32 [SL]
  static constexpr int A_QR = A_KS + SL * 4;                 // f16 [16][KROW] rotated q
  static constexpr int A_QW = A_QR + 16 * KROW * 2;          // bf16 [16][KROW] plain q
  static constexpr int A_LOG = A_QW + 16 * KROW * 2;         // fp32 [16][LST]
  static constexpr int A_P = A_LOG + 16 * LST * 4;           // f16 [16][PST]
  static constexpr int A_END = A_P + 16 * PST * 2;
  static_assert(A_QW >= S_END, "the query rows are copied in during the selection");
  static constexpr int REGION = ((A_END > S_END ? A_END : S_END) + 127) & ~127;

  static constexpr int OFF_WIN = REGION;                     // bf16 [WSL][kWRow] this CTA's window rows
  static constexpr int OFF_MERGE = OFF_WIN + WSL * kWRow;    // fp32 [CS][HPC][SLOT]
  // page-table entries of this CTA's 8192-block chunk (implicit sources)
  static constexpr int OFF_PT = OFF_MERGE + CS * HPC * SLOT * 4;  // i32 [kMaxKeys / kPage]
  static constexpr int OFF_SEL = OFF_PT + kMaxKeys / kPage * 4;  // i32 [256] positions
  static constexpr int OFF_OWN = OFF_SEL + kMaxTopK * 4;     // i32 [256] local block ids attended
  static constexpr int OFF_SCAN = OFF_OWN + kMaxTopK * 4;    // u32 [64]
  static constexpr int OFF_MISC = OFF_SCAN + 64 * 4;
  static constexpr int MISC_BYTES = 512;
  static constexpr int OFF_LUT = OFF_MISC + MISC_BYTES;      // u32 [256]: code byte -> half2
  static constexpr int OFF_CONST = OFF_LUT + 256 * 4;        // fp32 [128] rotation signs, [16] sinks
  static constexpr int SMEM = OFF_CONST + (kHeadDim + kMaxHeads) * 4;
  static_assert(SMEM <= 227 * 1024, "fits one CTA per SM");
};

// Score kernel: a CTA stages PPC index pages and scores them.
constexpr int kSThreads = 256;
constexpr int kSWarps = kSThreads / 32;
constexpr int kSU = 4;  // 16-key tiles a warp scores per loop iteration
template <int BITS>
struct SCfg {
  static constexpr int RB_IDX = kIdxDim * BITS / 8;
  static constexpr int PB_IDX = page_bytes(RB_IDX);
  static constexpr int PPC = BITS == 4 ? 16 : 8;  // pages per CTA (36 / 34 KB at 16 / 8)
  static constexpr int OFF_LIMB = PPC * PB_IDX;              // s8 [4 heads][3 limbs][64]
  static constexpr int OFF_MISC = OFF_LIMB + kIdxHeads * 3 * kIdxDim;
  static_assert(OFF_LIMB % 8 == 0, "limb rows are read 8 bytes at a time");
  static constexpr int OFF_BAR = OFF_MISC + 128;
  static constexpr int SMEM = OFF_BAR + 16;
  // codebook caches (csa_score_levels_kernel): rotated query fp32 [4][64],
  // level table fp32 [2^BITS]
  static constexpr int OFF_QROT = SMEM;
  static constexpr int OFF_LV = OFF_QROT + kIdxHeads * kIdxDim * 4;
  static constexpr int SMEM_LEVELS = OFF_LV + 256 * 4;
};

struct QParams {
  const float* levels;  // Lloyd-Max level table [2^bits] (codebook caches), or null (uniform codes)
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
  uint32_t* ws;    // [B][ws_stride] per-block score keys (kernel A -> kernel B)
  int ws_stride;
  // selection source of the attend kernel: the workspace row (implicit ids,
  // `chunks` CTAs per sequence each taking 8192 blocks) or an explicit
  // candidate list [B][cand_stride] of keys and ascending global ids
  int chunks;
  const uint32_t* cand_keys;
  const int32_t* cand_ids;
  int cand_n, cand_stride;
  // select-only output: top_k (key, id) per CTA, [B * chunks][top_k]
  uint32_t* sel_keys_out;
  int32_t* sel_ids_out;
  int sel_stride;  // row stride of the select-only output (multiple of 4)
  // this device holds blocks [id_base, id_base + nblocks[b]) of sequence b
  int id_base;
  // partial output for a cross-device merge: un-normalised O [B][H][128]
  // and (max logit, sum) [B][H][2]; the sink is left to the merge
  float* part_o;
  float* part_ml;
  // chunked prefill: query b reads page-table row q_row[b] and the window rows
  // win_row[b] .. win_row[b] + window_len[b] - 1 of a flat [rows][128] buffer
  // (null: row b, rows b * W ..)
  const int32_t* q_row;
  const long long* win_row;
  // optional inverse output RoPE (aether_2b/serving.py:469-472): rotate the
  // last rope_dim output channels by -rope_pos[b] with rope_inv_freq
  const int32_t* rope_pos;
  const float* rope_inv_freq;
  int rope_dim;
  // host-buffer steps on copy streams: step_flags[0] reaches step_seq once
  // this step's inputs are on the device, step_flags[1] reaches step_seq - 1
  // once the previous output copy from the same staging slot is done (null:
  // the stream orders both)
  const uint32_t* step_flags;
  uint32_t step_seq;
  long long* dbg;  // per-CTA phase timestamps [grid][16] (profiling aid), or null
  int* err;
  int table_stride, num_pages, H, W, top_k;
  float softmax_scale;
};

// workspace row stride (u32 keys): a multiple of 16 so rows are 64-byte aligned
__host__ __device__ inline int csa_workspace_stride(int max_nblocks) { return ((max_nblocks > 0 ? max_nblocks : 1) + 15) & ~15; }

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
  uint32_t nvalid;
  uint32_t nown;
  // selection rescale: smallest / largest valid key, smallest per-thread
  // maximum key, threads holding a valid key
  uint32_t kmin, kmax, tmin, nact;
  float m_h[kMaxHeads];
  float l_h[kMaxHeads];
};

// kr[j] for a run-time j < 16 without local memory (binary select tree)
__device__ __forceinline__ uint32_t pick16(const uint32_t (&kr)[16], int j) {
  uint32_t a[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) a[i] = (j & 1) ? kr[2 * i + 1] : kr[2 * i];
#pragma unroll
  for (int i = 0; i < 4; ++i) a[i] = (j & 2) ? a[2 * i + 1] : a[2 * i];
#pragma unroll
  for (int i = 0; i < 2; ++i) a[i] = (j & 4) ? a[2 * i + 1] : a[2 * i];
  return (j & 8) ? a[1] : a[0];
}

// Block-wide inclusive scan of one u32 per thread; uses wtot[0..63].
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
    wtot[32 + lane] = w;
  }
  __syncthreads();
  return (warp ? wtot[32 + warp - 1] : 0u) + inc;
}

// Bin holding the R-th largest element of a histogram scanned from the top
// bin down; writes bin, count above it and count in it to misc.
__device__ __forceinline__ void find_bin(const uint32_t* hist, int nbins, uint32_t R, uint32_t* wtot, QMisc* misc,
                                         int tid, int lane, int warp) {
  const int per = nbins / kQThreads;
  // thread tid owns the contiguous bins [nbins - per * (tid + 1), nbins - per * tid)
  uint32_t s = 0;
  const uint32_t* mine = hist + nbins - per * (tid + 1);
  if (per % 4 == 0) {
    for (int k = 0; k < per; k += 4) {
      const uint4 v = *reinterpret_cast<const uint4*>(mine + k);
      s += (v.x + v.y) + (v.z + v.w);
    }
  } else {
    for (int k = 0; k < per; ++k) s += mine[k];
  }
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

// histogram increment (lanes with bin < 0 do not count); plain shared
// atomics: on sm_100 they are far cheaper than warp-aggregation via match.any
__device__ __forceinline__ void hist_add(uint32_t* hist, int bin) {
  if (bin >= 0) atomicAdd(&hist[bin], 1u);
}

template <int BITS>
__global__ void __launch_bounds__(kSThreads) csa_score_kernel(QParams p, int splits) {
  using C = SCfg<BITS>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int b = blockIdx.x / splits, sp = blockIdx.x % splits;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  // profiling aid: phase timestamps after the attend kernel's area
  long long* dbg = p.dbg ? p.dbg + 65536 + blockIdx.x * 8 : nullptr;
  auto stamp = [&](int slot) {  // SM clock cycles (phase durations)
    if (dbg && tid == 0) dbg[slot] = clock64();
  };
  stamp(0);
  if (p.step_flags) {  // this step's inputs are copied on another stream
    if (tid == 0) flag_wait(p.step_flags, p.step_seq, p.err);
    __syncthreads();
  }
  pdl_launch_dependents();
  int nb = p.nblocks[b];
  nb = max(0, min(nb, min(kMaxBlocks, p.table_stride * kPage)));
  const int npages = (nb + kPage - 1) / kPage;
  const int pg0 = sp * C::PPC;
  if (pg0 >= npages) return;
  const int np = min(C::PPC, npages - pg0);
  int8_t* limb = reinterpret_cast<int8_t*>(smem + C::OFF_LIMB);
  float* alpha = reinterpret_cast<float*>(smem + C::OFF_MISC);
  int(*lsum)[3] = reinterpret_cast<int(*)[3]>(smem + C::OFF_MISC + 16);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  // the page table and the cache are state: stage the pages before waiting
  if (warp == 0) {
    if (lane == 0) mbar_expect_tx(bar, np * C::PB_IDX);
    __syncwarp();
    if (lane < np) {
      int phys = p.page_table[static_cast<long long>(b) * p.table_stride + pg0 + lane];
      if (phys < 0 || phys >= p.num_pages) {
        report_error(p.err, kErrBadPage);
        phys = 0;
      }
      bulk_g2s(smem + lane * C::PB_IDX, p.idx_pages + static_cast<long long>(phys) * C::PB_IDX, C::PB_IDX, bar);
    }
  }
  stamp(1);
  pdl_wait();
  if (warp < kIdxHeads) index_query_limbs(p.index_q, p.index_w, p.diag_idx, b, warp, lane, limb, alpha, lsum);
  __syncthreads();
  uint32_t bq[2][2][2];
  int c0i, c1i, c2i;
  limb_fragments<BITS>(limb, lsum, g, t, bq, c0i, c1i, c2i);
  const float alpha_t = alpha[t];
  stamp(2);
  mbar_wait(bar, 0, p.err);
  stamp(3);
  uint32_t* out = p.ws + static_cast<long long>(b) * p.ws_stride;
  const int tiles = np * (kPage / 16);
  for (int t0 = warp; t0 < tiles; t0 += kSU * kSWarps) {
    uint32_t a[kSU][2][4];
    int ra[kSU];
    bool ok[kSU];
#pragma unroll
    for (int u = 0; u < kSU; ++u) {
      const int tile = t0 + u * kSWarps;
      ok[u] = tile < tiles;
      const uint8_t* page = smem + (ok[u] ? (tile >> 2) : 0) * C::PB_IDX;
      ra[u] = (tile & 3) * 16 + g;
      if (BITS == 4) {
        const uint2 va = *reinterpret_cast<const uint2*>(page + ra[u] * C::RB_IDX + t * 8);
        const uint2 vb = *reinterpret_cast<const uint2*>(page + (ra[u] + 8) * C::RB_IDX + t * 8);
        a[u][0][0] = (va.x & 0x0F0F0F0Fu) ^ 0x08080808u;
        a[u][0][2] = ((va.x >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
        a[u][0][1] = (vb.x & 0x0F0F0F0Fu) ^ 0x08080808u;
        a[u][0][3] = ((vb.x >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
        a[u][1][0] = (va.y & 0x0F0F0F0Fu) ^ 0x08080808u;
        a[u][1][2] = ((va.y >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
        a[u][1][1] = (vb.y & 0x0F0F0F0Fu) ^ 0x08080808u;
        a[u][1][3] = ((vb.y >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
      } else {
        const uint4 va = *reinterpret_cast<const uint4*>(page + ra[u] * C::RB_IDX + t * 16);
        const uint4 vb = *reinterpret_cast<const uint4*>(page + (ra[u] + 8) * C::RB_IDX + t * 16);
        a[u][0][0] = va.x; a[u][0][1] = vb.x; a[u][0][2] = va.y; a[u][0][3] = vb.y;
        a[u][1][0] = va.z; a[u][1][1] = vb.z; a[u][1][2] = va.w; a[u][1][3] = vb.w;
      }
    }
    int acc0[kSU][4], acc1[kSU][4];
#pragma unroll
    for (int u = 0; u < kSU; ++u) {
      acc0[u][0] = c0i; acc0[u][1] = c1i; acc0[u][2] = c0i; acc0[u][3] = c1i;
      acc1[u][0] = c2i; acc1[u][1] = 0; acc1[u][2] = c2i; acc1[u][3] = 0;
    }
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int u = 0; u < kSU; ++u) {
        mma_s8(acc0[u], a[u][j][0], a[u][j][1], a[u][j][2], a[u][j][3], bq[0][j][0], bq[0][j][1]);
        mma_s8(acc1[u], a[u][j][0], a[u][j][1], a[u][j][2], a[u][j][3], bq[1][j][0], bq[1][j][1]);
      }
    // thread t holds head t: limbs (acc0[0], acc0[1], acc1[0]) for row a,
    // (acc0[2], acc0[3], acc1[2]) for row a + 8
    float sc[kSU][2];
#pragma unroll
    for (int u = 0; u < kSU; ++u)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const float d = __fadd_rn(__fmul_rn(static_cast<float>(acc1[u][2 * r]), 65536.f),
                                  __fadd_rn(__fmul_rn(static_cast<float>(acc0[u][2 * r + 1]), 256.f),
                                            static_cast<float>(acc0[u][2 * r])));
        sc[u][r] = alpha_t * fmaxf(d, 0.f);
      }
#pragma unroll
    for (int u = 0; u < kSU; ++u)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        sc[u][r] += __shfl_xor_sync(0xffffffffu, sc[u][r], 1);
        sc[u][r] += __shfl_xor_sync(0xffffffffu, sc[u][r], 2);
      }
#pragma unroll
    for (int u = 0; u < kSU; ++u) {
      const int tile = t0 + u * kSWarps;
      if (ok[u] && t < 2) {
        const uint8_t* page = smem + (tile >> 2) * C::PB_IDX;
        const float* ksc = reinterpret_cast<const float*>(page + kPage * C::RB_IDX);
        const int slot = ra[u] + 8 * t;
        const int key = (pg0 + (tile >> 2)) * kPage + slot;
        if (key < nb) {
          const float s = __fadd_rn(__fmul_rn(sc[u][t], ksc[slot]), 0.0f);
          out[key] = __float_as_uint(s) + 1u;  // order-preserving key, 0 = no block
        }
      }
    }
  }
  stamp(4);
}

// Score kernel for caches in the Lloyd-Max level format: a key's rotated
// entries are levels[c] * scale, so q_h . k_s = scale_s * (WHT(diag * q_h) .
// levels[c_s]) (aether_2b/modeling.py:609-611 with the keys decoded as
// levels, not integers).  The exact integer limb MMAs of csa_score_kernel do
// not apply to non-integer levels: fp32 FMAs instead, one index head per
// lane, the four heads of a key on the four lanes of a quad.  The same CTA
// shape, staging and key format as csa_score_kernel.
template <int BITS>
__global__ void __launch_bounds__(kSThreads) csa_score_levels_kernel(QParams p, int splits) {
  using C = SCfg<BITS>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int b = blockIdx.x / splits, sp = blockIdx.x % splits;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (p.step_flags) {  // this step's inputs are copied on another stream
    if (tid == 0) flag_wait(p.step_flags, p.step_seq, p.err);
    __syncthreads();
  }
  pdl_launch_dependents();
  int nb = p.nblocks[b];
  nb = max(0, min(nb, min(kMaxBlocks, p.table_stride * kPage)));
  const int npages = (nb + kPage - 1) / kPage;
  const int pg0 = sp * C::PPC;
  if (pg0 >= npages) return;
  const int np = min(C::PPC, npages - pg0);
  float* qrot = reinterpret_cast<float*>(smem + C::OFF_QROT);
  float* lv = reinterpret_cast<float*>(smem + C::OFF_LV);
  float* alpha = reinterpret_cast<float*>(smem + C::OFF_MISC);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == 0) {  // the pages are cache state: staged before the wait
    if (lane == 0) mbar_expect_tx(bar, np * C::PB_IDX);
    __syncwarp();
    if (lane < np) {
      int phys = p.page_table[static_cast<long long>(b) * p.table_stride + pg0 + lane];
      if (phys < 0 || phys >= p.num_pages) {
        report_error(p.err, kErrBadPage);
        phys = 0;
      }
      bulk_g2s(smem + lane * C::PB_IDX, p.idx_pages + static_cast<long long>(phys) * C::PB_IDX, C::PB_IDX, bar);
    }
  }
  pdl_wait();
  if (tid < (1 << BITS)) lv[tid] = p.levels[tid];
  if (warp < kIdxHeads) {
    float v0, v1;
    rotate_index_query(p.index_q, p.diag_idx, b, warp, lane, v0, v1);
    qrot[warp * kIdxDim + 2 * lane] = v0;
    qrot[warp * kIdxDim + 2 * lane + 1] = v1;
    if (lane == 0) alpha[warp] = softplus_f(p.index_w[b * kIdxHeads + warp]);
  }
  __syncthreads();
  const int h = lane & 3;
  float qr[kIdxDim];
#pragma unroll
  for (int d = 0; d < kIdxDim; ++d) qr[d] = qrot[h * kIdxDim + d];
  const float a_h = alpha[h];
  mbar_wait(bar, 0, p.err);
  uint32_t* out = p.ws + static_cast<long long>(b) * p.ws_stride;
  // a quad per key: every pass covers 64 keys, so every lane of a quad runs
  // the same passes
  for (int key = tid >> 2; key < np * kPage; key += kSThreads / 4) {
    const uint8_t* page = smem + (key >> 6) * C::PB_IDX;
    const int slot = key & 63;
    const uint8_t* row = page + slot * C::RB_IDX;
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < C::RB_IDX; c += 4) {
      const uint32_t w = *reinterpret_cast<const uint32_t*>(row + c);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t byte = (w >> (8 * e)) & 0xFFu;
        if (BITS == 4) {
          dot = fmaf(qr[2 * (c + e)], lv[byte & 15u], dot);
          dot = fmaf(qr[2 * (c + e) + 1], lv[byte >> 4], dot);
        } else {
          dot = fmaf(qr[c + e], lv[byte], dot);
        }
      }
    }
    float sc = a_h * fmaxf(dot, 0.f);
    sc += __shfl_xor_sync(0xffffffffu, sc, 1);
    sc += __shfl_xor_sync(0xffffffffu, sc, 2);
    const int gk = (pg0 + (key >> 6)) * kPage + slot;
    if (h == 0 && gk < nb) {
      const float ks = reinterpret_cast<const float*>(page + kPage * C::RB_IDX)[slot];
      out[gk] = __float_as_uint(__fadd_rn(__fmul_rn(sc, ks), 0.0f)) + 1u;  // order-preserving key
    }
  }
}

template <int BITS, int CS>
__global__ void __launch_bounds__(kQThreads, CS > 1 ? 2 : 1) csa_attend_kernel(QParams p) {
  using C = QCfg<BITS, CS>;
  extern __shared__ __align__(128) uint8_t smem[];
  // grid: ((sequence * chunks) + chunk) * CS + rank; a cluster of CS CTAs
  // serves one (sequence, chunk): every CTA selects, each attends a slice
  const int r = blockIdx.x % CS;
  const int bc = blockIdx.x / CS;
  const int b = bc / p.chunks, chunk = bc % p.chunks;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const bool select_only = p.sel_keys_out != nullptr;
  auto stamp = [&](int slot, bool who) {  // SM clock cycles (phase durations)
    if (p.dbg && who) p.dbg[blockIdx.x * 16 + slot] = clock64();
  };
  stamp(0, tid == 0);
  pdl_launch_dependents();
  // announce this CTA is running; the wait comes before the first remote access
  if constexpr (CS > 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");

  uint8_t* winb = smem + C::OFF_WIN;
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem + C::S_HIST);
  float* merge = reinterpret_cast<float*>(smem + C::OFF_MERGE);
  int32_t* pt = reinterpret_cast<int32_t*>(smem + C::OFF_PT);
  int32_t* sel = reinterpret_cast<int32_t*>(smem + C::OFF_SEL);
  int32_t* own = reinterpret_cast<int32_t*>(smem + C::OFF_OWN);
  uint32_t* wtot = reinterpret_cast<uint32_t*>(smem + C::OFF_SCAN);
  QMisc* misc = reinterpret_cast<QMisc*>(smem + C::OFF_MISC);
  uint32_t* lut = reinterpret_cast<uint32_t*>(smem + C::OFF_LUT);
  if ((BITS == 4 || p.levels) && tid < 256) lut[tid] = code_lut_entry(BITS, p.levels, static_cast<uint32_t>(tid));

  // ------------------------------------------------------------ prologue
  int nb = p.nblocks[b];  // blocks of sequence b held on this device
  if (nb > kMaxBlocks || nb > p.table_stride * kPage) {
    if (tid == 0) report_error(p.err, kErrBadShape);
    nb = min(kMaxBlocks, p.table_stride * kPage);
  }
  nb = max(nb, 0);
  const bool explicit_list = p.cand_keys != nullptr;
  // keys this CTA selects from: positions 0..n-1, in ascending block-id order
  const int n = explicit_list ? min(p.cand_n, kMaxKeys) : max(0, min(nb - chunk * kMaxKeys, kMaxKeys));
  const int npages = (nb + kPage - 1) / kPage;
  const int W = p.W;
  const int wl = select_only ? 0 : max(0, min(p.window_len[b], W));
  const long long wbase = p.win_row ? p.win_row[b] : static_cast<long long>(b) * W;  // first window row
  const int wsl = (W + CS - 1) / CS;               // window rows per CTA
  const int w0 = r * wsl;                           // this CTA's first window row
  const int wn = max(0, min(wl - w0, wsl));         // its valid window rows
  // implicit sources lie in this CTA's chunk: stage its page-table entries;
  // explicit candidate lists may name any block, read at the gather
  const int32_t* ptab = p.page_table + static_cast<long long>(p.q_row ? p.q_row[b] : b) * p.table_stride;
  const int pt0 = chunk * (kMaxKeys / kPage);
  if (!select_only && !explicit_list) {
    for (int i = tid; i < min(npages - pt0, kMaxKeys / kPage); i += kQThreads) {
      int v = ptab[pt0 + i];
      if (v < 0 || v >= p.num_pages) {
        report_error(p.err, kErrBadPage);
        v = 0;
      }
      pt[i] = v;
    }
  }
  // with at most top_k candidate positions every valid key is taken: no
  // histogram (prefill's explicit top-k lists, short contexts)
  const bool need_select = n > p.top_k;
  if (need_select)
    for (int i = tid; i < kL1Bins / 4; i += kQThreads) reinterpret_cast<uint4*>(hist)[i] = make_uint4(0, 0, 0, 0);
  if (tid < kMaxTopK) sel[tid] = 0;  // every slot holds a valid position
  if (tid == 0) {
    misc->thr = 0;
    misc->take_eq = 0xFFFFFFFFu;
    misc->bin = 0;
    misc->above = 0;
    misc->cnt = 0;
    misc->nvalid = 0;
    misc->nown = 0;
    misc->ncand = 0;
    misc->kmin = 0xFFFFFFFFu;
    misc->kmax = 0;
    misc->tmin = 0xFFFFFFFFu;
    misc->nact = 0;
  }
  // window rows other than the newest are cache state: prefetch them now
  {
    const int pre = max(0, min(wn, wl - 1 - w0));
    const __nv_bfloat16* wsrc = p.window + (wbase + w0) * kHeadDim;
    for (int i = tid; i < pre * 16; i += kQThreads)
      cp_async16(winb + (i >> 4) * kWRow + (i & 15) * 16, wsrc + (i >> 4) * kHeadDim + (i & 15) * 8);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  // model constants read late in the chain, staged now so their global-load
  // latency is not paid there: the rotation signs and the sinks
  if (!select_only) {
    float* cst = reinterpret_cast<float*>(smem + C::OFF_CONST);
    if (tid < kHeadDim) cst[tid] = __ldg(p.diag_kv + tid);
    if (!p.part_o && tid < p.H) cst[kHeadDim + tid] = __ldg(p.sink + tid);
  }
  // the block keys come from the score kernel (or a previous select)
  pdl_wait();
  // the staging slot's previous output copy must be done before this step's
  // stores (the __syncthreads below orders the other threads)
  if (p.step_flags && tid == 0) flag_wait(p.step_flags + 1, p.step_seq - 1u, p.err);
  // this warp's query head (a step input, so after the wait) is copied into
  // its plain-query row now: the load latency overlaps the selection instead
  // of the gather (the row lies outside the selection's shared area)
  if (!select_only) {
    if (warp < p.H)
      cp_async8(smem + C::A_QW + (warp * C::KROW + lane * 4) * 2,
                p.q + (static_cast<long long>(b) * p.H + warp) * kHeadDim + lane * 4);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  stamp(2, tid == 0);
  // a short explicit list that needs no selection (prefill's top-k lists):
  // one candidate per thread; the winners are the valid keys in list order
  const bool few = explicit_list && !select_only && n <= kQThreads && n <= p.top_k;
  int ko_direct = -1;  // winners attended, when every thread knows it without a barrier
  if (few) {
    const uint32_t* ck = p.cand_keys + static_cast<long long>(b) * p.cand_stride;
    const int32_t* ci = p.cand_ids + static_cast<long long>(b) * p.cand_stride;
    const uint32_t key = tid < n ? __ldcg(ck + tid) : 0u;
    const int gid = tid < n ? __ldcg(ci + tid) : -1;
    const bool valid = key != 0u;
    const int loc = valid && gid >= p.id_base && gid < p.id_base + nb ? gid - p.id_base : -1;
    const uint32_t bv = __ballot_sync(0xffffffffu, valid), bo = __ballot_sync(0xffffffffu, loc >= 0);
    if (lane == 0) {
      wtot[warp] = __popc(bv);
      wtot[32 + warp] = __popc(bo);
    }
    __syncthreads();
    uint32_t pv = 0, po = 0, tv = 0, to = 0;
    for (int w = 0; w < kQWarps; ++w) {
      const uint32_t cv = wtot[w], co = wtot[32 + w];
      if (w < warp) {
        pv += cv;
        po += co;
      }
      tv += cv;
      to += co;
    }
    const uint32_t lt = (1u << lane) - 1u;
    if (loc >= 0) own[po + __popc(bo & lt)] = loc;
    if (p.sel_out && r == 0) {
      int32_t* so = p.sel_out + static_cast<long long>(b) * p.top_k;
      if (valid) so[pv + __popc(bv & lt)] = gid;
      for (int i = static_cast<int>(tv) + tid; i < p.top_k; i += kQThreads) so[i] = -1;
    }
    if (tid == 0) misc->nown = to;
    stamp(5, tid == 0);
  } else {
    constexpr int PER = kMaxKeys / kQThreads;  // 16 keys per thread, in source order
    const int i0 = tid * PER;
    uint32_t kr[PER];
    {
      const uint32_t* src = explicit_list ? p.cand_keys + static_cast<long long>(b) * p.cand_stride + i0
                                          : p.ws + static_cast<long long>(b) * p.ws_stride + chunk * kMaxKeys + i0;
  #pragma unroll
      for (int v = 0; v < PER / 4; ++v) {
        uint4 x = make_uint4(0, 0, 0, 0);
        if (i0 + 4 * v < n) x = __ldcg(reinterpret_cast<const uint4*>(src) + v);
        kr[4 * v] = x.x; kr[4 * v + 1] = x.y; kr[4 * v + 2] = x.z; kr[4 * v + 3] = x.w;
      }
    }
    // the prologue's zero-fill of the histogram and of misc happens-before
    // any update (the key loads above are already in flight)
    __syncthreads();
    {
      uint32_t cnt = 0, lo = 0xFFFFFFFFu, hi = 0;
  #pragma unroll
      for (int j = 0; j < PER; ++j) {
        kr[j] = i0 + j < n ? kr[j] : 0u;  // key 0 = no block
        if (kr[j]) {
          ++cnt;
          lo = min(lo, kr[j]);
          hi = max(hi, kr[j]);
        }
      }
      const uint32_t tmax = hi;
      cnt = __reduce_add_sync(0xffffffffu, cnt);
      uint32_t tlo = 0, nact = 0;
      if (need_select) {
        lo = __reduce_min_sync(0xffffffffu, lo);
        hi = __reduce_max_sync(0xffffffffu, hi);
        tlo = __reduce_min_sync(0xffffffffu, tmax ? tmax : 0xFFFFFFFFu);
        nact = __popc(__ballot_sync(0xffffffffu, tmax != 0u));
      }
      if (lane == 0 && cnt) {
        atomicAdd(&misc->nvalid, cnt);
        if (need_select) {
          atomicMin(&misc->kmin, lo);
          atomicMax(&misc->kmax, hi);
          atomicMin(&misc->tmin, tlo);
          atomicAdd(&misc->nact, nact);
        }
      }
    }
    __syncthreads();
    if (p.score_out && !explicit_list && r == 0) {
      float* so = p.score_out + static_cast<long long>(b) * p.score_stride + chunk * kMaxKeys + i0;
  #pragma unroll
      for (int j = 0; j < PER; ++j)
        if (i0 + j < n) so[j] = __uint_as_float(kr[j] - 1u);
    }
    if (need_select) {
      // Rescale the keys before binning.  lo is a lower bound of the K-th
      // largest key: when at least K threads hold a valid key, the smallest
      // per-thread maximum (each of those threads holds a key >= it), else
      // the smallest key.  Keys >= lo map to (k - lo + 2) << z, z chosen so
      // the largest stays below 2^31 (bins of key >> 19 stay < 4096): a
      // strictly increasing map.  Keys < lo are never taken and all map to 1,
      // below every mapped key >= lo.  So the selected set, its ties and their
      // position order are unchanged, while the band [lo, kmax] -- a narrow
      // range of float exponents -- spreads over all 4096 top-level bins and
      // the boundary bin holds a key or two instead of dozens.
      const uint32_t kq = static_cast<uint32_t>(min(p.top_k, static_cast<int>(misc->nvalid)));
      const uint32_t lo = misc->nact >= kq ? misc->tmin : misc->kmin;
      const int z = __clz(misc->kmax - lo + 2u) - 1;
  #pragma unroll
      for (int j = 0; j < PER; ++j)
        if (kr[j]) {
          kr[j] = kr[j] >= lo ? (kr[j] - lo + 2u) << z : 1u;
          atomicAdd(&hist[kr[j] >> 19], 1u);
        }
      __syncthreads();
    }
    stamp(3, tid == 0);
    const int nvalid = static_cast<int>(misc->nvalid);
    const int K = min(p.top_k, nvalid);

    // ------------------------------------------------------------- select
    // Result: every key > thr is taken, and the take_eq lowest-position keys
    // == thr.  Keys are >= 1 for real blocks, so thr = 0 takes all of them.
    // After the bin b1 of the K-th largest key (bins of key >> 19) is known,
    // later steps walk `wmask`, the bit set of this thread's keys in bins >= b1.
    uint32_t wmask = 0;
  #pragma unroll
    for (int j = 0; j < PER; ++j) wmask |= static_cast<uint32_t>(kr[j] != 0u) << j;
    if (nvalid > K) {
      find_bin(hist, kL1Bins, static_cast<uint32_t>(K), wtot, misc, tid, lane, warp);
      const uint32_t b1 = misc->bin, ccnt = misc->cnt;
      const uint32_t R = static_cast<uint32_t>(K) - misc->above;  // keys still to take from bin b1
      wmask = 0;
  #pragma unroll
      for (int j = 0; j < PER; ++j) wmask |= static_cast<uint32_t>(kr[j] != 0u && (kr[j] >> 19) >= b1) << j;
      if (ccnt == R) {
        if (tid == 0) misc->thr = b1 << 19;  // lowest key of bin b1: the whole bin is taken
      } else if (ccnt <= static_cast<uint32_t>(kBoundMax)) {
        // rank the keys of bin b1 exactly: (key desc, position asc)
        uint2* cand = reinterpret_cast<uint2*>(hist + kL1Bins);
        for (uint32_t m = wmask; m; m &= m - 1u) {
          const int j = __ffs(m) - 1;
          const uint32_t kj = pick16(kr, j);
          if ((kj >> 19) == b1) cand[atomicAdd(&misc->ncand, 1u)] = make_uint2(kj, i0 + j);
        }
        __syncthreads();
        for (int i = tid; i < static_cast<int>(ccnt); i += kQThreads) {
          const uint2 me = cand[i];
          uint32_t rank = 0, eq_before = 0;
          for (int k2 = 0; k2 < static_cast<int>(ccnt); ++k2) {
            const uint2 o = cand[k2];
            rank += o.x > me.x || (o.x == me.x && o.y < me.y);
            eq_before += o.x == me.x && o.y < me.y;
          }
          if (rank == R - 1) {  // the last key taken
            misc->thr = me.x;
            misc->take_eq = eq_before + 1;
          }
        }
      } else {
        // many keys share bin b1: two more radix levels over those keys
        uint32_t R2 = R;
        for (int i = tid; i < 2048; i += kQThreads) hist[i] = 0;
        __syncthreads();
        for (uint32_t m = wmask; m; m &= m - 1u) {
          const uint32_t kj = pick16(kr, __ffs(m) - 1);
          if ((kj >> 19) == b1) atomicAdd(&hist[(kj >> 8) & 2047u], 1u);
        }
        __syncthreads();
        find_bin(hist, 2048, R2, wtot, misc, tid, lane, warp);
        const uint32_t b2 = misc->bin;
        R2 -= misc->above;
        const uint32_t pfx = (b1 << 11) | b2;  // key >> 8
        if (misc->cnt == R2) {
          if (tid == 0) misc->thr = pfx << 8;  // the whole sub-bin is taken
        } else {
          for (int i = tid; i < kQThreads; i += kQThreads) hist[i] = 0;
          __syncthreads();
          for (uint32_t m = wmask; m; m &= m - 1u) {
            const uint32_t kj = pick16(kr, __ffs(m) - 1);
            if ((kj >> 8) == pfx) atomicAdd(&hist[kj & 255u], 1u);
          }
          __syncthreads();
          find_bin(hist, kQThreads, R2, wtot, misc, tid, lane, warp);  // 256 used bins of 512
          R2 -= misc->above;
          if (tid == 0) {
            misc->thr = (pfx << 8) | static_cast<uint32_t>(misc->bin);
            misc->take_eq = R2;  // keys equal to thr: the lowest-position R2 of them
          }
        }
      }
    }
    __syncthreads();
    stamp(4, tid == 0);
    // ordered compaction over wmask: thread order is source order.  On the
    // implicit (single-device, in-order) source every winner is held here, so
    // the attended list `own` is written directly.
    const bool direct_own = !explicit_list && p.id_base == 0 && !select_only;
    {
      const uint32_t thr = misc->thr, take_eq = misc->take_eq;
      uint32_t cs = 0, ce = 0;
      for (uint32_t m = wmask; m; m &= m - 1u) {
        const uint32_t kj = pick16(kr, __ffs(m) - 1);
        cs += kj > thr;
        ce += kj == thr;
      }
      const uint32_t packed = cs | (ce << 16);
      const uint32_t exc = block_scan_incl(packed, wtot, lane, warp) - packed;
      uint32_t sb = exc & 0xFFFFu, eb = exc >> 16;  // 16-bit fields: at most 8192 keys
      for (uint32_t m = (cs | ce) ? wmask : 0u; m; m &= m - 1u) {
        const int j = __ffs(m) - 1;
        const uint32_t kj = pick16(kr, j);
        const bool st = kj > thr, eq = kj == thr;
        const uint32_t pos = st ? sb + min(eb, take_eq) : sb + eb;
        if ((st || (eq && eb < take_eq)) && pos < static_cast<uint32_t>(K)) {
          sel[pos] = i0 + j;
          if (direct_own) own[pos] = chunk * kMaxKeys + i0 + j;
        }
        sb += st;
        eb += eq;
      }
    }
    __syncthreads();
    stamp(5, tid == 0);
    // global block id of a source position
    const int32_t* cids = explicit_list ? p.cand_ids + static_cast<long long>(b) * p.cand_stride : nullptr;
    auto gid_of = [&](int pos) -> int { return explicit_list ? cids[pos] : p.id_base + chunk * kMaxKeys + pos; };
    if (select_only) {
      if (r == 0) {
        const uint32_t* kk = explicit_list ? p.cand_keys + static_cast<long long>(b) * p.cand_stride
                                           : p.ws + static_cast<long long>(b) * p.ws_stride + chunk * kMaxKeys;
        const long long o = static_cast<long long>(bc) * p.sel_stride;
        for (int i = tid; i < p.sel_stride; i += kQThreads) {
          p.sel_keys_out[o + i] = i < K ? __ldcg(kk + sel[i]) : 0u;
          p.sel_ids_out[o + i] = i < K ? gid_of(sel[i]) : -1;
        }
      }
      return;
    }
    if (p.sel_out && r == 0) {
      int32_t* so = p.sel_out + static_cast<long long>(b) * p.top_k;
      for (int i = tid; i < p.top_k; i += kQThreads) so[i] = i < K ? gid_of(sel[i]) : -1;
    }
    // the selected blocks held on this device, as local ids (order kept)
    if (direct_own) {
      ko_direct = K;  // own[] is complete at the compaction's barrier
    } else {
      // thread i < K looks up winner i (all id loads in flight together); a
      // ballot per warp and the per-warp counts keep the winners' order
      int loc = -1;
      if (tid < K) {
        const int gidv = gid_of(sel[tid]);
        if (gidv >= p.id_base && gidv < p.id_base + nb) loc = gidv - p.id_base;
      }
      const uint32_t bal = __ballot_sync(0xffffffffu, loc >= 0);
      constexpr int kSelWarps = kMaxTopK / 32;
      if (lane == 0 && warp < kSelWarps) wtot[warp] = __popc(bal);
      __syncthreads();
      if (warp < kSelWarps) {
        uint32_t base = 0;
        for (int w = 0; w < warp; ++w) base += wtot[w];
        if (loc >= 0) own[base + __popc(bal & ((1u << lane) - 1))] = loc;
        if (tid == 0) {
          uint32_t tot = 0;
          for (int w = 0; w < kSelWarps; ++w) tot += wtot[w];
          misc->nown = tot;
        }
      }
    }
  }
  if (ko_direct < 0) __syncthreads();  // CTA-uniform condition
  const int KO = ko_direct >= 0 ? ko_direct : static_cast<int>(misc->nown);
  // this CTA's slice of the winners
  const int slc = (((KO + CS - 1) / CS) + 15) & ~15;
  const int s0 = min(KO, r * slc);
  const int kc = max(0, min(KO - s0, slc));

  // --------------------------------------------------------- attention
  __half* Kc = reinterpret_cast<__half*>(smem + C::A_KC);
  float* ks = reinterpret_cast<float*>(smem + C::A_KS);
  __half* Qr = reinterpret_cast<__half*>(smem + C::A_QR);
  __nv_bfloat16* Qw = reinterpret_cast<__nv_bfloat16*>(smem + C::A_QW);
  float* logit = reinterpret_cast<float*>(smem + C::A_LOG);
  __half* P = reinterpret_cast<__half*>(smem + C::A_P);
  const int ntc = (kc + 15) / 16, ntw = (wn + 15) / 16;
  // winners' code rows and scales straight into registers (expanded to fp16
  // below, after the query work, once the loads have landed)
  constexpr int CPR = C::RB_KV / 16;
  constexpr int NCH = (C::SL * CPR + kQThreads - 1) / kQThreads;
  uint4 cw[NCH];
  float csc[NCH];
  {
#pragma unroll
    for (int u = 0; u < NCH; ++u) {
      const int i = tid + u * kQThreads;
      cw[u] = make_uint4(0, 0, 0, 0);
      csc[u] = 0.f;
      if (i >= kc * CPR) continue;
      const int row = i / CPR, ch = i % CPR;
      const int blk = min(max(own[s0 + row], 0), max(nb - 1, 0));
      int phys;
      if (explicit_list) {
        phys = __ldg(ptab + (blk >> 6));
        if (phys < 0 || phys >= p.num_pages) {
          report_error(p.err, kErrBadPage);
          phys = 0;
        }
      } else {
        phys = pt[min(max((blk >> 6) - pt0, 0), kMaxKeys / kPage - 1)];
      }
      const uint8_t* pg = p.kv_pages + static_cast<long long>(phys) * C::PB_KV;
      cw[u] = *reinterpret_cast<const uint4*>(pg + (blk & 63) * C::RB_KV + ch * 16);
      if (ch == 0) csc[u] = *reinterpret_cast<const float*>(pg + kPage * C::RB_KV + (blk & 63) * 4);
    }
    // newest window row (written by the previous step), if it is in this slice
    if (wl > 0 && wl - 1 >= w0 && wl - 1 < w0 + wsl && tid < 16)
      cp_async16(winb + (wl - 1 - w0) * kWRow + tid * 16,
                 p.window + (wbase + wl - 1) * kHeadDim + tid * 8);
  }
  // queries: plain bf16 rows for the window, rotated fp16 rows for the codes
  {
    const int h = warp;  // 16 warps, 16 padded heads
    float v[4];
    if (h < p.H) {
      // committed groups only: the query row (the newest window row's copy is
      // not committed yet); each lane waits for its own copy, the warp then shares
      asm volatile("cp.async.wait_group 0;" ::: "memory");
      __syncwarp();
      const uint2 r4 = *reinterpret_cast<const uint2*>(Qw + h * C::KROW + lane * 4);
      const __nv_bfloat162* bb = reinterpret_cast<const __nv_bfloat162*>(&r4);
      const float2 f0 = __bfloat1622float2(bb[0]), f1 = __bfloat1622float2(bb[1]);
      v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
    } else {
      *reinterpret_cast<uint2*>(Qw + h * C::KROW + lane * 4) = make_uint2(0, 0);
      v[0] = v[1] = v[2] = v[3] = 0.f;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] *= reinterpret_cast<const float*>(smem + C::OFF_CONST)[lane * 4 + k];
    warp_wht128(v, lane);
    const float cn = 0.0883883461356163f;
    *reinterpret_cast<uint2*>(Qr + h * C::KROW + lane * 4) =
        make_uint2(pack_half2(v[0] * cn, v[1] * cn), pack_half2(v[2] * cn, v[3] * cn));
  }
  // zero window rows past wn up to the tile edge
  for (int i = tid; i < (ntw * 16 - wn) * 16; i += kQThreads)
    *reinterpret_cast<uint4*>(winb + (wn + (i >> 4)) * kWRow + (i & 15) * 16) = make_uint4(0, 0, 0, 0);
  // codes -> exact fp16 rows; rows past kc zero-filled to the tile edge
#pragma unroll
  for (int u = 0; u < NCH; ++u) {
    const int i = tid + u * kQThreads;
    if (i >= kc * CPR) continue;
    const int row = i / CPR, ch = i % CPR;
    if (ch == 0) ks[row] = csc[u];
    const uint32_t wd[4] = {cw[u].x, cw[u].y, cw[u].z, cw[u].w};
    if (BITS == 4) {
      __half* dst = Kc + row * C::KROW + ch * 32;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t w = wd[k];
        *reinterpret_cast<uint4*>(dst + k * 8) =
            make_uint4(lut[w & 0xFFu], lut[(w >> 8) & 0xFFu], lut[(w >> 16) & 0xFFu], lut[w >> 24]);
      }
    } else {
      __half* dst = Kc + row * C::KROW + ch * 16;
      const bool lv = p.levels != nullptr;
#pragma unroll
      for (int k = 0; k < 2; ++k)
        *reinterpret_cast<uint4*>(dst + k * 8) =
            make_uint4(code8_pair(wd[2 * k], lut, lv), code8_pair(wd[2 * k] >> 16, lut, lv),
                       code8_pair(wd[2 * k + 1], lut, lv), code8_pair(wd[2 * k + 1] >> 16, lut, lv));
    }
  }
  for (int i = tid; i < (ntc * 16 - kc) * 16; i += kQThreads) {
    const int row = kc + (i >> 4);
    *reinterpret_cast<uint4*>(Kc + row * C::KROW + (i & 15) * 8) = make_uint4(0, 0, 0, 0);
    if ((i & 15) == 0) ks[row] = 0.f;
  }
  cp_async_commit_wait_all();
  __syncthreads();
  stamp(6, tid == 0);

  // ---- S = Q K^T, one 16-source tile per warp iteration
  for (int tile = warp; tile < ntc + ntw; tile += kQWarps) {
    const bool comp = tile < ntc;
    float acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
    float acc2[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
    if (comp) {
      const __half* Kt = Kc + tile * 16 * C::KROW;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t a[4], b0, b1, b2, b3;
        ldsm_x4(a[0], a[1], a[2], a[3], Qr + (lane & 15) * C::KROW + kk * 16 + (lane >> 4) * 8);
        ldsm_x4(b0, b1, b2, b3, Kt + ((lane & 7) + ((lane >> 4) << 3)) * C::KROW + kk * 16 + ((lane >> 3) & 1) * 8);
        mma_f16((kk & 1) ? acc2[0] : acc[0], a, b0, b1);
        mma_f16((kk & 1) ? acc2[1] : acc[1], a, b2, b3);
      }
    } else {
      const uint8_t* wt = winb + (tile - ntc) * 16 * kWRow;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t a[4], b0, b1, b2, b3;
        ldsm_x4(a[0], a[1], a[2], a[3], Qw + (lane & 15) * C::KROW + kk * 16 + (lane >> 4) * 8);
        ldsm_x4(b0, b1, b2, b3, wt + ((lane & 7) + ((lane >> 4) << 3)) * kWRow + (kk * 16 + ((lane >> 3) & 1) * 8) * 2);
        mma_bf16((kk & 1) ? acc2[0] : acc[0], a, b0, b1);
        mma_bf16((kk & 1) ? acc2[1] : acc[1], a, b2, b3);
      }
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int h = g + (e >> 1) * 8;
        const int src = tile * 16 + nt * 8 + 2 * t;
        float z0 = acc[nt][e] + acc2[nt][e], z1 = acc[nt][e + 1] + acc2[nt][e + 1];
        if (comp) {
          z0 = src < kc ? z0 * ks[src] * p.softmax_scale : -INFINITY;
          z1 = src + 1 < kc ? z1 * ks[src + 1] * p.softmax_scale : -INFINITY;
        } else {
          z0 = (src - ntc * 16) < wn ? z0 * p.softmax_scale : -INFINITY;
          z1 = (src + 1 - ntc * 16) < wn ? z1 * p.softmax_scale : -INFINITY;
        }
        *reinterpret_cast<float2*>(logit + h * C::LST + src) = make_float2(z0, z1);
      }
  }
  __syncthreads();
  stamp(7, tid == 0);
  // ---- softmax statistics, one warp per head, 4 columns per lane step
  const int ncols = (ntc + ntw) * 16, ncc = ntc * 16;
  if (warp >= p.H) {
    for (int c = lane * 4; c < ncols; c += 128) *reinterpret_cast<uint2*>(P + warp * C::PST + c) = make_uint2(0, 0);
  } else {
    const int h = warp;
    float m = -INFINITY;
    for (int c = lane * 4; c < ncols; c += 128) {
      const float4 z = *reinterpret_cast<const float4*>(logit + h * C::LST + c);
      m = fmaxf(m, fmaxf(fmaxf(z.x, z.y), fmaxf(z.z, z.w)));
    }
    m = warp_max(m);
    const float mu = m == -INFINITY ? 0.f : m;
    float l = 0.f;
    for (int c = lane * 4; c < ncols; c += 128) {
      const float4 z = *reinterpret_cast<const float4*>(logit + h * C::LST + c);
      const float e0 = __expf(z.x - mu), e1 = __expf(z.y - mu), e2 = __expf(z.z - mu), e3 = __expf(z.w - mu);
      l += (e0 + e1) + (e2 + e3);
      float4 w = make_float4(e0, e1, e2, e3);
      if (c < ncc) {  // compressed columns carry the per-entry scale into P
        const float4 s4 = *reinterpret_cast<const float4*>(ks + c);
        w = make_float4(e0 * s4.x, e1 * s4.y, e2 * s4.z, e3 * s4.w);
      }
      *reinterpret_cast<uint2*>(P + h * C::PST + c) = make_uint2(pack_half2(w.x, w.y), pack_half2(w.z, w.w));
    }
    l = warp_sum(l);
    if (lane == 0) {
      misc->m_h[h] = m;
      misc->l_h[h] = l;
    }
  }
  __syncthreads();
  stamp(8, tid == 0);
  // ---- O = P V.  Warps 0-7 take the compressed tiles, warps 8-15 the
  // window tiles, each warp output dims [16 (w % 8), +16): every warp reads
  // only its own part of P (P is every warp's A operand; its shared-memory
  // reads, not the MMAs, bound this phase) and the two parts land in
  // separate fields of the merge slot.  Partials go to the head's owner CTA
  // (slot r), which merges them
  {
    static_assert(kQWarps == 16, "P V split: 16 warps");
    const int dg = warp & 7;
    const bool win_part = warp >= 8;
    float o[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
    const int vr = (lane & 7) + ((lane >> 3) & 1) * 8, vc = dg * 16 + (lane >> 4) * 8;  // x4.trans source
    if (!win_part) {
      for (int kt = 0; kt < ntc; ++kt) {
        uint32_t a[4], bb[4];
        ldsm_x4(a[0], a[1], a[2], a[3], P + (lane & 15) * C::PST + kt * 16 + (lane >> 4) * 8);
        ldsm_x4_t(bb[0], bb[1], bb[2], bb[3], Kc + (kt * 16 + vr) * C::KROW + vc);
        mma_f16(o[0], a, bb[0], bb[1]);
        mma_f16(o[1], a, bb[2], bb[3]);
      }
    } else {
      for (int kt = ntc; kt < ntc + ntw; ++kt) {
        uint32_t a[4], bb[4];
        ldsm_x4(a[0], a[1], a[2], a[3], P + (lane & 15) * C::PST + kt * 16 + (lane >> 4) * 8);
        ldsm_x4_t(bb[0], bb[1], bb[2], bb[3], winb + ((kt - ntc) * 16 + vr) * kWRow + vc * 2);
        mma_f16(o[0], a, bf2_to_h2(bb[0]), bf2_to_h2(bb[1]));
        mma_f16(o[1], a, bf2_to_h2(bb[2]), bf2_to_h2(bb[3]));
      }
    }
    const int hpc = (p.H + CS - 1) / CS;
    if constexpr (CS > 1) asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      const int h = g + (e >> 1) * 8;
      if (h < p.H) {
        const int owner = h / hpc, lh = h % hpc;
        float* slot = merge + (r * C::HPC + lh) * C::SLOT;
        if constexpr (CS > 1) slot = cg::this_cluster().map_shared_rank(slot, owner);
        slot += 4 + (win_part ? kHeadDim : 0);
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
          *reinterpret_cast<float2*>(slot + dg * 16 + nt * 8 + 2 * t) = make_float2(o[nt][e], o[nt][e + 1]);
      }
    }
  }
  if (warp == 0 && lane < p.H) {
    const int hpc = (p.H + CS - 1) / CS;
    const int h = lane, owner = h / hpc, lh = h % hpc;
    float* slot = merge + (r * C::HPC + lh) * C::SLOT;
    if constexpr (CS > 1) slot = cg::this_cluster().map_shared_rank(slot, owner);
    slot[0] = misc->m_h[h];
    slot[1] = misc->l_h[h];
  }
  if constexpr (CS > 1) cg::this_cluster().sync();
  else __syncthreads();
  stamp(9, tid == 0);

  // ---- owner: merge the CS partials of its heads, inverse rotation, then
  // the final sink-normalised bf16 output or the partial (O, max, sum)
  {
    const int hpc = (p.H + CS - 1) / CS;
    for (int lh = warp; lh < hpc; lh += kQWarps) {
      const int h = r * hpc + lh;
      if (h >= p.H) break;
      float M = -INFINITY;
#pragma unroll
      for (int rr = 0; rr < CS; ++rr) M = fmaxf(M, merge[(rr * C::HPC + lh) * C::SLOT]);
      float L = 0.f, vr[4] = {0, 0, 0, 0}, vw[4] = {0, 0, 0, 0};
#pragma unroll
      for (int rr = 0; rr < CS; ++rr) {
        const float* slot = merge + (rr * C::HPC + lh) * C::SLOT;
        const float m = slot[0];
        const float a = m == -INFINITY ? 0.f : __expf(m - M);
        L += a * slot[1];
        const float4 o1 = *reinterpret_cast<const float4*>(slot + 4 + lane * 4);
        const float4 o2 = *reinterpret_cast<const float4*>(slot + 4 + kHeadDim + lane * 4);
        vr[0] += a * o1.x; vr[1] += a * o1.y; vr[2] += a * o1.z; vr[3] += a * o1.w;
        vw[0] += a * o2.x; vw[1] += a * o2.y; vw[2] += a * o2.z; vw[3] += a * o2.w;
      }
      warp_wht128(vr, lane);
      float o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) o[k] = vr[k] * 0.0883883461356163f * reinterpret_cast<const float*>(smem + C::OFF_CONST)[lane * 4 + k] + vw[k];
      if (p.part_o) {
        *reinterpret_cast<float4*>(p.part_o + (static_cast<long long>(b) * p.H + h) * kHeadDim + lane * 4) =
            make_float4(o[0], o[1], o[2], o[3]);
        if (lane == 0)
          *reinterpret_cast<float2*>(p.part_ml + (static_cast<long long>(b) * p.H + h) * 2) = make_float2(M, L);
      } else {
        const float sk = reinterpret_cast<const float*>(smem + C::OFF_CONST)[kHeadDim + h];
        const float Ms = fmaxf(M, sk);
        const float a = M == -INFINITY ? 0.f : __expf(M - Ms);
        const float inv = a / (L * a + __expf(sk - Ms));
#pragma unroll
        for (int k = 0; k < 4; ++k) o[k] *= inv;
        if (p.rope_inv_freq) {
          const float pos = static_cast<float>(-p.rope_pos[b]);
          const int first = kHeadDim - p.rope_dim;
#pragma unroll
          for (int k = 0; k < 4; k += 2) {
            const int dd = lane * 4 + k;  // even channel of the pair (dd, dd + 1)
            if (dd >= first) {
              const float ang = pos * p.rope_inv_freq[(dd - first) >> 1];
              const float cs = cosf(ang), sn = sinf(ang);
              const float x0 = o[k], x1 = o[k + 1];
              o[k] = x0 * cs - x1 * sn;
              o[k + 1] = x1 * cs + x0 * sn;
            }
          }
        }
        __nv_bfloat162 o01 = __floats2bfloat162_rn(o[0], o[1]);
        __nv_bfloat162 o23 = __floats2bfloat162_rn(o[2], o[3]);
        *reinterpret_cast<uint2*>(p.out + (static_cast<long long>(b) * p.H + h) * kHeadDim + lane * 4) =
            make_uint2(*reinterpret_cast<uint32_t*>(&o01), *reinterpret_cast<uint32_t*>(&o23));
      }
    }
  }
  stamp(10, tid == 0);
}

// ======================================================================
// HCA decode (modeling.py:384-410, serving.py:507-522): every visible
// compressed block plus the sliding window, no selection.  A 4-CTA cluster
// per sequence; CTA r attends blocks [256 r, 256 r + 256) (four whole pages)
// and window rows [w0, w0 + 32).  Everything that is cache state -- the page
// table, the pages (one bulk copy each), their fp16 expansion and every
// window row but the newest -- is staged before griddepcontrol.wait, so under
// programmatic dependent launch it overlaps the previous kernel; after the
// wait only the query-dependent work runs: rotated query, S = Q K^T, softmax,
// O = P V, and the DSMEM merge of the four partials with the sink.
constexpr int kHcaCS = 4;
constexpr int kHcaRows = 256;                   // compressed rows per CTA
constexpr int kHcaPages = kHcaRows / kPage;     // 4
constexpr int kHcaMaxBlocks = kHcaCS * kHcaRows;  // 1024 (131072 tokens at compression 128)

template <int BITS>
struct HCfg {
  static constexpr int RB_KV = kHeadDim * BITS / 8;
  static constexpr int PB_KV = page_bytes(RB_KV);
  static constexpr int KROW = kHeadDim + 8;                 // fp16 operand row stride (halves)
  static constexpr int WSL = kWinMax / kHcaCS;              // window rows per CTA (max)
  static constexpr int LST = kHcaRows + WSL + 8;            // logit row stride (floats), = 8 mod 32
  static constexpr int PST = kHcaRows + WSL + 8;            // P row stride (halves)
  static constexpr int HPC = kMaxHeads / kHcaCS;            // heads finalised per CTA (max)
  static constexpr int SLOT = 4 + 2 * kHeadDim;             // merge slot: m, l, pad, pad, O_rot, O_win
  static constexpr int A_KC = 0;                            // f16 [256][KROW] expanded codes
  static constexpr int A_KS = A_KC + kHcaRows * KROW * 2;   // fp32 [256] row scales
  static constexpr int A_QR = A_KS + kHcaRows * 4;          // f16 [16][KROW] rotated q
  static constexpr int A_QW = A_QR + 16 * KROW * 2;         // bf16 [16][KROW] plain q
  // the staged pages are dead once expanded: logits and P reuse their space
  static constexpr int A_RAW = A_QW + 16 * KROW * 2;        // [4] pages
  static constexpr int A_LOG = A_RAW;                       // fp32 [16][LST]
  static constexpr int A_P = A_LOG + 16 * LST * 4;          // f16 [16][PST]
  static constexpr int RAW_END = A_RAW + kHcaPages * PB_KV;
  static constexpr int P_END = A_P + 16 * PST * 2;
  static constexpr int OFF_WIN = ((RAW_END > P_END ? RAW_END : P_END) + 127) & ~127;  // bf16 [WSL][kWRow]
  static constexpr int OFF_MERGE = OFF_WIN + WSL * kWRow;   // fp32 [CS][HPC][SLOT]
  static constexpr int OFF_MISC = OFF_MERGE + kHcaCS * HPC * SLOT * 4;  // m_h[16], l_h[16]
  static constexpr int OFF_LUT = OFF_MISC + 2 * kMaxHeads * 4;          // u32 [256]: code byte -> half2
  static constexpr int OFF_BAR = OFF_LUT + 256 * 4;        // u64 [4]: one per staged page
  static constexpr int OFF_CONST = OFF_BAR + 8 * kHcaPages;  // fp32 [128] rotation signs, [16] sinks
  static constexpr int SMEM = OFF_CONST + (kHeadDim + kMaxHeads) * 4;
  static_assert(A_RAW % 128 == 0 && PB_KV % 16 == 0, "bulk-copy destinations are 16-byte aligned");
  static_assert(SMEM <= 227 * 1024, "fits one CTA per SM");
};

struct HcaParams {
  const float* levels;          // Lloyd-Max level table [2^bits], or null (uniform codes)
  const __nv_bfloat16* q;       // [B, H, 128]
  const float* sink;            // [H]
  const __nv_bfloat16* window;  // [B, W, 128]
  const int32_t* window_len;    // [B]
  const uint8_t* kv_pages;      // [P][64 x 128*bits/8 codes | 64 x fp32 scales]
  const int32_t* page_table;    // [B, table_stride]
  const int32_t* nblocks;       // [B]
  const float* diag_kv;         // [128] +-1
  __nv_bfloat16* out;           // [B, H, 128]
  long long* dbg;
  int* err;
  int table_stride, num_pages, H, W;
  float softmax_scale;
};

template <int BITS>
__global__ void __launch_bounds__(kQThreads, 1) hca_attend_kernel(HcaParams p) {
  using C = HCfg<BITS>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int r = blockIdx.x % kHcaCS, b = blockIdx.x / kHcaCS;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  auto stamp = [&](int slot) {  // SM clock cycles (phase durations)
    if (p.dbg && tid == 0) p.dbg[blockIdx.x * 16 + slot] = clock64();
  };
  stamp(0);
  pdl_launch_dependents();
  // announce this CTA is running; the wait comes before the first remote store
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");

  __half* Kc = reinterpret_cast<__half*>(smem + C::A_KC);
  float* ks = reinterpret_cast<float*>(smem + C::A_KS);
  __half* Qr = reinterpret_cast<__half*>(smem + C::A_QR);
  __nv_bfloat16* Qw = reinterpret_cast<__nv_bfloat16*>(smem + C::A_QW);
  uint8_t* raw = smem + C::A_RAW;
  float* logit = reinterpret_cast<float*>(smem + C::A_LOG);
  __half* P = reinterpret_cast<__half*>(smem + C::A_P);
  uint8_t* winb = smem + C::OFF_WIN;
  float* merge = reinterpret_cast<float*>(smem + C::OFF_MERGE);
  float* m_h = reinterpret_cast<float*>(smem + C::OFF_MISC);
  float* l_h = m_h + kMaxHeads;
  uint32_t* lut = reinterpret_cast<uint32_t*>(smem + C::OFF_LUT);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);

  // ------------------------------------------- prologue: cache state only
  // independent loads first: block count, window length, this CTA's four
  // page-table entries
  const int32_t* ptab = p.page_table + static_cast<long long>(b) * p.table_stride + r * kHcaPages;
  int phys = 0;
  if (warp == 0 && lane < kHcaPages && r * kHcaPages + lane < p.table_stride) phys = ptab[lane];
  int nb = p.nblocks[b];
  const int wl_raw = p.window_len[b];
  if (nb > kHcaMaxBlocks || nb > p.table_stride * kPage) {
    if (tid == 0) report_error(p.err, kErrBadShape);
    nb = min(kHcaMaxBlocks, p.table_stride * kPage);
  }
  nb = max(nb, 0);
  const int kc = max(0, min(nb - r * kHcaRows, kHcaRows));  // this CTA's compressed rows
  const int npg = (kc + kPage - 1) / kPage;
  const int W = p.W;
  const int wl = max(0, min(wl_raw, W));
  const int wsl = (W + kHcaCS - 1) / kHcaCS;
  const int w0 = r * wsl;
  const int wn = max(0, min(wl - w0, wsl));  // this CTA's window rows
  const int ntc = (kc + 15) / 16, ntw = (wn + 15) / 16;
  // one mbarrier per page, initialised and armed by the issuing warp
  if (warp == 0) {
    if (lane < kHcaPages) mbar_init(bar + lane, 1);
    fence_mbar_init();
    __syncwarp();
    if (lane < npg) {
      if (phys < 0 || phys >= p.num_pages) {
        report_error(p.err, kErrBadPage);
        phys = 0;
      }
      mbar_expect_tx(bar + lane, C::PB_KV);
      bulk_g2s(raw + lane * C::PB_KV, p.kv_pages + static_cast<long long>(phys) * C::PB_KV, C::PB_KV, bar + lane);
    }
  }
  if ((BITS == 4 || p.levels) && tid < 256) lut[tid] = code_lut_entry(BITS, p.levels, static_cast<uint32_t>(tid));
  // model constants (rotation signs, sinks) staged with the cache state
  {
    float* cst = reinterpret_cast<float*>(smem + C::OFF_CONST);
    if (tid < kHeadDim) cst[tid] = __ldg(p.diag_kv + tid);
    if (tid < p.H) cst[kHeadDim + tid] = __ldg(p.sink + tid);
  }
  // window rows other than the newest are cache state
  const long long wbase = static_cast<long long>(b) * W;
  {
    const int pre = max(0, min(wn, wl - 1 - w0));
    const __nv_bfloat16* wsrc = p.window + (wbase + w0) * kHeadDim;
    for (int i = tid; i < pre * 16; i += kQThreads)
      cp_async16(winb + (i >> 4) * kWRow + (i & 15) * 16, wsrc + (i >> 4) * kHeadDim + (i & 15) * 8);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  // zero window rows past wn up to the tile edge
  for (int i = tid; i < (ntw * 16 - wn) * 16; i += kQThreads)
    *reinterpret_cast<uint4*>(winb + (wn + (i >> 4)) * kWRow + (i & 15) * 16) = make_uint4(0, 0, 0, 0);
  __syncthreads();  // barriers initialised, LUT written
  stamp(1);
  // codes -> exact fp16 rows, scales -> ks, page by page as each lands (rows
  // past kc zero to the tile edge)
  for (int pg = 0; pg * kPage < ntc * 16; ++pg) {
    if (pg < npg) mbar_wait(bar + pg, 0, p.err);
    const uint8_t* src = raw + pg * C::PB_KV;
    for (int i = tid; i < kPage * 16; i += kQThreads) {
      const int prow = i >> 4, row = pg * kPage + prow, c8 = (i & 15) * 8;
      if (row >= ntc * 16) break;
      uint4 o = make_uint4(0, 0, 0, 0);
      if (row < kc) {
        if (BITS == 4) {
          const uint32_t w = *reinterpret_cast<const uint32_t*>(src + prow * C::RB_KV + c8 / 2);
          o = make_uint4(lut[w & 0xFFu], lut[(w >> 8) & 0xFFu], lut[(w >> 16) & 0xFFu], lut[w >> 24]);
        } else {
          const uint2 w = *reinterpret_cast<const uint2*>(src + prow * C::RB_KV + c8);
          const bool lv = p.levels != nullptr;
          o = make_uint4(code8_pair(w.x, lut, lv), code8_pair(w.x >> 16, lut, lv), code8_pair(w.y, lut, lv),
                         code8_pair(w.y >> 16, lut, lv));
        }
      }
      if ((i & 15) == 0)
        ks[row] = row < kc ? *reinterpret_cast<const float*>(src + kPage * C::RB_KV + prow * 4) : 0.f;
      *reinterpret_cast<uint4*>(Kc + row * C::KROW + c8) = o;
    }
  }
  stamp(2);

  // ------------------------------------------- query-dependent work
  pdl_wait();
  stamp(3);
  {
    const int h = warp;  // 16 warps, 16 padded heads
    float v[4];
    if (h < p.H) {
      const uint2 r4 = *reinterpret_cast<const uint2*>(p.q + (static_cast<long long>(b) * p.H + h) * kHeadDim + lane * 4);
      *reinterpret_cast<uint2*>(Qw + h * C::KROW + lane * 4) = r4;
      const __nv_bfloat162* bb = reinterpret_cast<const __nv_bfloat162*>(&r4);
      const float2 f0 = __bfloat1622float2(bb[0]), f1 = __bfloat1622float2(bb[1]);
      v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
    } else {
      *reinterpret_cast<uint2*>(Qw + h * C::KROW + lane * 4) = make_uint2(0, 0);
      v[0] = v[1] = v[2] = v[3] = 0.f;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] *= reinterpret_cast<const float*>(smem + C::OFF_CONST)[lane * 4 + k];
    warp_wht128(v, lane);
    const float cn = 0.0883883461356163f;
    *reinterpret_cast<uint2*>(Qr + h * C::KROW + lane * 4) =
        make_uint2(pack_half2(v[0] * cn, v[1] * cn), pack_half2(v[2] * cn, v[3] * cn));
  }
  // the newest window row (written by the previous kernel)
  if (wl > 0 && wl - 1 >= w0 && wl - 1 < w0 + wn && tid < 16)
    cp_async16(winb + (wl - 1 - w0) * kWRow + tid * 16, p.window + (wbase + wl - 1) * kHeadDim + tid * 8);
  cp_async_commit_wait_all();
  __syncthreads();
  stamp(4);

  // ---- S = Q K^T, one 16-source tile per warp iteration; the rotated
  // query's A fragments stay in registers
  uint32_t qa[8][4];
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    ldsm_x4(qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], Qr + (lane & 15) * C::KROW + kk * 16 + (lane >> 4) * 8);
  for (int tile = warp; tile < ntc + ntw; tile += kQWarps) {
    const bool comp = tile < ntc;
    float acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
    float acc2[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
    if (comp) {
      const __half* Kt = Kc + tile * 16 * C::KROW;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(b0, b1, b2, b3, Kt + ((lane & 7) + ((lane >> 4) << 3)) * C::KROW + kk * 16 + ((lane >> 3) & 1) * 8);
        mma_f16((kk & 1) ? acc2[0] : acc[0], qa[kk], b0, b1);
        mma_f16((kk & 1) ? acc2[1] : acc[1], qa[kk], b2, b3);
      }
    } else {
      const uint8_t* wt = winb + (tile - ntc) * 16 * kWRow;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t a[4], b0, b1, b2, b3;
        ldsm_x4(a[0], a[1], a[2], a[3], Qw + (lane & 15) * C::KROW + kk * 16 + (lane >> 4) * 8);
        ldsm_x4(b0, b1, b2, b3, wt + ((lane & 7) + ((lane >> 4) << 3)) * kWRow + (kk * 16 + ((lane >> 3) & 1) * 8) * 2);
        mma_bf16((kk & 1) ? acc2[0] : acc[0], a, b0, b1);
        mma_bf16((kk & 1) ? acc2[1] : acc[1], a, b2, b3);
      }
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int h = g + (e >> 1) * 8;
        const int src = tile * 16 + nt * 8 + 2 * t;
        float z0 = acc[nt][e] + acc2[nt][e], z1 = acc[nt][e + 1] + acc2[nt][e + 1];
        if (comp) {
          z0 = src < kc ? z0 * ks[src] * p.softmax_scale : -INFINITY;
          z1 = src + 1 < kc ? z1 * ks[src + 1] * p.softmax_scale : -INFINITY;
        } else {
          z0 = (src - ntc * 16) < wn ? z0 * p.softmax_scale : -INFINITY;
          z1 = (src + 1 - ntc * 16) < wn ? z1 * p.softmax_scale : -INFINITY;
        }
        *reinterpret_cast<float2*>(logit + h * C::LST + src) = make_float2(z0, z1);
      }
  }
  __syncthreads();
  stamp(5);
  // ---- softmax statistics, one warp per head, 4 columns per lane step
  const int ncols = (ntc + ntw) * 16, ncc = ntc * 16;
  if (warp >= p.H) {
    for (int c = lane * 4; c < ncols; c += 128) *reinterpret_cast<uint2*>(P + warp * C::PST + c) = make_uint2(0, 0);
  } else {
    const int h = warp;
    float m = -INFINITY;
    for (int c = lane * 4; c < ncols; c += 128) {
      const float4 z = *reinterpret_cast<const float4*>(logit + h * C::LST + c);
      m = fmaxf(m, fmaxf(fmaxf(z.x, z.y), fmaxf(z.z, z.w)));
    }
    m = warp_max(m);
    const float mu = m == -INFINITY ? 0.f : m;
    float l = 0.f;
    for (int c = lane * 4; c < ncols; c += 128) {
      const float4 z = *reinterpret_cast<const float4*>(logit + h * C::LST + c);
      const float e0 = __expf(z.x - mu), e1 = __expf(z.y - mu), e2 = __expf(z.z - mu), e3 = __expf(z.w - mu);
      l += (e0 + e1) + (e2 + e3);
      float4 w = make_float4(e0, e1, e2, e3);
      if (c < ncc) {  // compressed columns carry the per-entry scale into P
        const float4 s4 = *reinterpret_cast<const float4*>(ks + c);
        w = make_float4(e0 * s4.x, e1 * s4.y, e2 * s4.z, e3 * s4.w);
      }
      *reinterpret_cast<uint2*>(P + h * C::PST + c) = make_uint2(pack_half2(w.x, w.y), pack_half2(w.z, w.w));
    }
    l = warp_sum(l);
    if (lane == 0) {
      m_h[h] = m;
      l_h[h] = l;
    }
  }
  __syncthreads();
  stamp(6);
  // ---- O = P V; warp w owns output dims [16 (w % 8), +16) over the 16-row
  // tiles of parity w / 8, so each warp reads half of P (P is every warp's A
  // operand: shared-memory reads of P, not the MMAs, bound this phase); the
  // odd-parity half is added through the dead logit area, then the sums go to
  // the head's owner CTA, which merges them
  const int hpc = (p.H + kHcaCS - 1) / kHcaCS;
  {
    static_assert(kQWarps == 16 && 16 * C::LST >= 8 * 32 * 16, "P V split: 16 warps, exchange fits the logits");
    const int dg = warp & 7, kh = warp >> 3;
    float orot[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}}, owin[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
    const int vr = (lane & 7) + ((lane >> 3) & 1) * 8, vc = dg * 16 + (lane >> 4) * 8;  // x4.trans source
    for (int kt = kh; kt < ntc; kt += 2) {
      uint32_t a[4], b[4];
      ldsm_x4(a[0], a[1], a[2], a[3], P + (lane & 15) * C::PST + kt * 16 + (lane >> 4) * 8);
      ldsm_x4_t(b[0], b[1], b[2], b[3], Kc + (kt * 16 + vr) * C::KROW + vc);
      mma_f16(orot[0], a, b[0], b[1]);
      mma_f16(orot[1], a, b[2], b[3]);
    }
    for (int kt = ntc + kh; kt < ntc + ntw; kt += 2) {
      uint32_t a[4], b[4];
      ldsm_x4(a[0], a[1], a[2], a[3], P + (lane & 15) * C::PST + kt * 16 + (lane >> 4) * 8);
      ldsm_x4_t(b[0], b[1], b[2], b[3], winb + ((kt - ntc) * 16 + vr) * kWRow + vc * 2);
      mma_f16(owin[0], a, bf2_to_h2(b[0]), bf2_to_h2(b[1]));
      mma_f16(owin[1], a, bf2_to_h2(b[2]), bf2_to_h2(b[3]));
    }
    float4* xh = reinterpret_cast<float4*>(logit) + (dg * 32 + lane) * 4;  // [8 dim groups][32 lanes][16 floats]
    if (kh == 1) {
      xh[0] = make_float4(orot[0][0], orot[0][1], orot[0][2], orot[0][3]);
      xh[1] = make_float4(orot[1][0], orot[1][1], orot[1][2], orot[1][3]);
      xh[2] = make_float4(owin[0][0], owin[0][1], owin[0][2], owin[0][3]);
      xh[3] = make_float4(owin[1][0], owin[1][1], owin[1][2], owin[1][3]);
    }
    __syncthreads();
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
    if (kh == 0) {
      float4 x[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) x[i] = xh[i];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        orot[nt][0] += x[nt].x; orot[nt][1] += x[nt].y; orot[nt][2] += x[nt].z; orot[nt][3] += x[nt].w;
        owin[nt][0] += x[2 + nt].x; owin[nt][1] += x[2 + nt].y; owin[nt][2] += x[2 + nt].z; owin[nt][3] += x[2 + nt].w;
      }
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int h = g + (e >> 1) * 8;
        if (h < p.H) {
          const int owner = h / hpc, lh = h % hpc;
          float* slot = cg::this_cluster().map_shared_rank(merge + (r * C::HPC + lh) * C::SLOT, owner);
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            const int dd = dg * 16 + nt * 8 + 2 * t;
            *reinterpret_cast<float2*>(slot + 4 + dd) = make_float2(orot[nt][e], orot[nt][e + 1]);
            *reinterpret_cast<float2*>(slot + 4 + kHeadDim + dd) = make_float2(owin[nt][e], owin[nt][e + 1]);
          }
        }
      }
    }
  }
  if (warp == 0 && lane < p.H) {
    const int h = lane, owner = h / hpc, lh = h % hpc;
    float* slot = cg::this_cluster().map_shared_rank(merge + (r * C::HPC + lh) * C::SLOT, owner);
    slot[0] = m_h[h];
    slot[1] = l_h[h];
  }
  cg::this_cluster().sync();
  stamp(7);
  // ---- owner: merge the four partials of its heads with the sink, inverse
  // rotation of the compressed part, bf16 store
  for (int lh = warp; lh < hpc; lh += kQWarps) {
    const int h = r * hpc + lh;
    if (h >= p.H) break;
    const float sk = reinterpret_cast<const float*>(smem + C::OFF_CONST)[kHeadDim + h];
    float M = sk;
#pragma unroll
    for (int rr = 0; rr < kHcaCS; ++rr) M = fmaxf(M, merge[(rr * C::HPC + lh) * C::SLOT]);
    float L = __expf(sk - M), vr[4] = {0, 0, 0, 0}, vw[4] = {0, 0, 0, 0};
#pragma unroll
    for (int rr = 0; rr < kHcaCS; ++rr) {
      const float* slot = merge + (rr * C::HPC + lh) * C::SLOT;
      const float m = slot[0];
      const float a = m == -INFINITY ? 0.f : __expf(m - M);
      L += a * slot[1];
      const float4 o1 = *reinterpret_cast<const float4*>(slot + 4 + lane * 4);
      const float4 o2 = *reinterpret_cast<const float4*>(slot + 4 + kHeadDim + lane * 4);
      vr[0] += a * o1.x; vr[1] += a * o1.y; vr[2] += a * o1.z; vr[3] += a * o1.w;
      vw[0] += a * o2.x; vw[1] += a * o2.y; vw[2] += a * o2.z; vw[3] += a * o2.w;
    }
    warp_wht128(vr, lane);
    const float inv = 1.f / L;
    float o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = (vr[k] * 0.0883883461356163f * reinterpret_cast<const float*>(smem + C::OFF_CONST)[lane * 4 + k] + vw[k]) * inv;
    __nv_bfloat162 o01 = __floats2bfloat162_rn(o[0], o[1]), o23 = __floats2bfloat162_rn(o[2], o[3]);
    *reinterpret_cast<uint2*>(p.out + (static_cast<long long>(b) * p.H + h) * kHeadDim + lane * 4) =
        make_uint2(*reinterpret_cast<uint32_t*>(&o01), *reinterpret_cast<uint32_t*>(&o23));
  }
  stamp(8);
}

constexpr int kAttendCluster = 2;  // CTAs per sequence in the attention phase

// Dynamic shared memory that keeps a second attend CTA off an SM.  The
// attend CTA needs ~99 KB, so two fit on one SM; when a launch's CTAs fit the
// GPU one per SM (decode batches), requesting this much spreads them over all
// SMs instead of pairing them on half of them, which halves each CTA's
// latency-bound phases.  Larger launches (prefill) use the compact size.
constexpr int kSpreadSmem = 116 * 1024;

static int sm_count() {  // of the current device
  int dev = 0, v = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    return 148;
  }
  return v;
}

template <int BITS>
static int set_smem_attrs() {
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(csa_score_kernel<BITS>), SCfg<BITS>::SMEM,
                            "csa_decode (score)");
  if (!rc)
    rc = ensure_smem_attr(reinterpret_cast<const void*>(csa_score_levels_kernel<BITS>), SCfg<BITS>::SMEM_LEVELS,
                          "csa_decode (score, level table)");
  if (!rc)
    rc = ensure_smem_attr(reinterpret_cast<const void*>(csa_attend_kernel<BITS, 1>), QCfg<BITS, 1>::SMEM,
                          "csa_decode (select)");
  if (!rc)
    rc = ensure_smem_attr(reinterpret_cast<const void*>(csa_attend_kernel<BITS, kAttendCluster>),
                          QCfg<BITS, kAttendCluster>::SMEM > kSpreadSmem ? QCfg<BITS, kAttendCluster>::SMEM
                                                                          : kSpreadSmem,
                          "csa_decode (attend)");
  return rc;
}

template <int BITS>
static int launch_score(const QParams& p, int B, int max_nblocks, bool pdl, cudaStream_t st) {
  using CA = SCfg<BITS>;
  const int max_pages = (max_nblocks + kPage - 1) / kPage;
  const int splits = max(1, (max_pages + CA::PPC - 1) / CA::PPC);
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t c = {};
  c.gridDim = dim3(B * splits);
  c.blockDim = dim3(kSThreads);
  c.dynamicSmemBytes = p.levels ? CA::SMEM_LEVELS : CA::SMEM;
  c.stream = st;
  c.attrs = at;
  c.numAttrs = pdl ? 1 : 0;
  if (p.levels)
    AETHER_CUDA_TRY(cudaLaunchKernelEx(&c, csa_score_levels_kernel<BITS>, p, splits), "csa_decode: launch (score)");
  else
    AETHER_CUDA_TRY(cudaLaunchKernelEx(&c, csa_score_kernel<BITS>, p, splits), "csa_decode: launch (score)");
  return 0;
}

// select-only launches use single CTAs; attention launches a cluster per sequence
template <int BITS>
static int launch_attend(const QParams& p, int B, bool pdl, cudaStream_t st) {
  const bool sel_only = p.sel_keys_out != nullptr;
  const int cs = sel_only ? 1 : kAttendCluster;
  cudaLaunchAttribute at[2];
  int na = 0;
  if (pdl) {
    at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (cs > 1) {
    at[na].id = cudaLaunchAttributeClusterDimension;
    at[na].val.clusterDim.x = cs;
    at[na].val.clusterDim.y = 1;
    at[na].val.clusterDim.z = 1;
    ++na;
  }
  cudaLaunchConfig_t c = {};
  c.gridDim = dim3(B * p.chunks * cs);
  c.blockDim = dim3(kQThreads);
  c.stream = st;
  c.attrs = at;
  c.numAttrs = na;
  if (sel_only) {
    c.dynamicSmemBytes = QCfg<BITS, 1>::SMEM;
    AETHER_CUDA_TRY(cudaLaunchKernelEx(&c, csa_attend_kernel<BITS, 1>, p), "csa_decode: launch (select)");
  } else {
    const int grid = B * p.chunks * cs;
    c.dynamicSmemBytes = grid <= sm_count() && QCfg<BITS, kAttendCluster>::SMEM < kSpreadSmem
                             ? kSpreadSmem
                             : QCfg<BITS, kAttendCluster>::SMEM;
    AETHER_CUDA_TRY(cudaLaunchKernelEx(&c, csa_attend_kernel<BITS, kAttendCluster>, p), "csa_decode: launch (attend)");
  }
  return 0;
}

static long long* g_cta_debug = nullptr;

// workspace layout: u32 keys [B][ws_stride], then candidate keys / ids
// [B][chunks * kMaxTopK] each (only for sequences longer than 8192 blocks)
static size_t workspace_bytes(int B, int max_nblocks) {
  const size_t keys = static_cast<size_t>(B) * csa_workspace_stride(max_nblocks) * 4;
  const int chunks = (max_nblocks + kMaxKeys - 1) / kMaxKeys;
  const size_t cand = chunks > 1 ? static_cast<size_t>(B) * chunks * kMaxTopK * 8 : 0;  // sel_stride <= 256
  return keys + cand;
}

static int check_common(int bits, int H, int W, int top_k, int max_nblocks, int table_stride, int num_pages) {
  AETHER_REQUIRE(bits == 4 || bits == 8, "bits must be 4 or 8, got %d", bits);
  AETHER_REQUIRE(H >= 1 && H <= kMaxHeads, "num_heads must be in [1, %d], got %d", kMaxHeads, H);
  AETHER_REQUIRE(W >= 0 && W <= kWinMax, "window capacity must be in [0, %d], got %d", kWinMax, W);
  AETHER_REQUIRE(top_k >= 1 && top_k <= kMaxTopK, "top_k must be in [1, %d], got %d", kMaxTopK, top_k);
  AETHER_REQUIRE(max_nblocks >= 0 && max_nblocks <= kMaxBlocks,
                 "csa decode: %d visible blocks exceed the per-device limit %d", max_nblocks, kMaxBlocks);
  AETHER_REQUIRE(table_stride >= 1 && num_pages >= 1, "page table / pool must be non-empty");
  return 0;
}

static QParams base_params(const void* q, const float* index_q, const float* index_w, const float* sink,
                           const void* window, const int32_t* window_len, const uint8_t* idx_pages,
                           const uint8_t* kv_pages, const int32_t* page_table, int table_stride, int num_pages,
                           const int32_t* nblocks, int max_nblocks, const float* diag_idx, const float* diag_kv,
                           int H, int W, int top_k, float softmax_scale, int* err) {
  QParams p{};
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
  p.ws_stride = csa_workspace_stride(max_nblocks);
  p.chunks = 1;
  p.dbg = g_cta_debug;
  p.err = err;
  p.table_stride = table_stride;
  p.num_pages = num_pages;
  p.H = H;
  p.W = W;
  p.top_k = top_k;
  p.softmax_scale = softmax_scale;
  return p;
}

template <int BITS>
static int run_decode(QParams p, int B, int max_nblocks, bool pdl, cudaStream_t st, uint8_t* workspace) {
  int rc = set_smem_attrs<BITS>();
  if (rc) return rc;
  p.ws = reinterpret_cast<uint32_t*>(workspace);
  const int chunks = (max_nblocks + kMaxKeys - 1) / kMaxKeys;
  rc = launch_score<BITS>(p, B, max_nblocks, pdl, st);
  if (rc) return rc;
  if (chunks <= 1) return launch_attend<BITS>(p, B, true, st);
  // long sequences: top-k per 8192-block chunk, then top-k of the chunk winners
  uint32_t* ckeys = p.ws + static_cast<size_t>(B) * p.ws_stride;
  int32_t* cids = reinterpret_cast<int32_t*>(ckeys + static_cast<size_t>(B) * chunks * kMaxTopK);
  QParams ps = p;
  ps.chunks = chunks;
  ps.sel_keys_out = ckeys;
  ps.sel_ids_out = cids;
  ps.out = nullptr;
  ps.sel_out = nullptr;
  ps.score_out = nullptr;
  ps.sel_stride = (p.top_k + 3) & ~3;
  // candidate rows are laid out [B * chunks][sel_stride]; reread as [B][chunks * sel_stride]
  rc = launch_attend<BITS>(ps, B, true, st);
  if (rc) return rc;
  QParams pa = p;
  pa.cand_keys = ckeys;
  pa.cand_ids = cids;
  pa.cand_n = chunks * ps.sel_stride;
  pa.cand_stride = chunks * ps.sel_stride;
  pa.score_out = nullptr;
  return launch_attend<BITS>(pa, B, true, st);
}

// HCA decode with the 4-CTA cluster kernel; pdl: programmatic dependent launch.
int hca_decode_cta(const void* q, const float* sink, const void* window, const int32_t* window_len,
                   const uint8_t* kv_pages, const int32_t* page_table, int table_stride, int num_pages,
                   const int32_t* nblocks, int max_nblocks, const float* diag_kv, int B, int H, int W, int bits,
                   float softmax_scale, void* out, int* err, int pdl, void* stream, const float* levels) {
  AETHER_REQUIRE(bits == 4 || bits == 8, "bits must be 4 or 8, got %d", bits);
  AETHER_REQUIRE(H >= 1 && H <= kMaxHeads, "num_heads must be in [1, %d], got %d", kMaxHeads, H);
  AETHER_REQUIRE(W >= 0 && W <= kWinMax, "window capacity must be in [0, %d], got %d", kWinMax, W);
  AETHER_REQUIRE(B >= 0, "batch must be non-negative");
  AETHER_REQUIRE(table_stride >= 1 && num_pages >= 1, "page table / pool must be non-empty");
  AETHER_REQUIRE(max_nblocks <= kHcaMaxBlocks, "hca decode: %d visible blocks exceed the limit %d", max_nblocks,
                 kHcaMaxBlocks);
  AETHER_REQUIRE(q && sink && window && window_len && kv_pages && page_table && nblocks && diag_kv && out,
                 "hca decode: null argument");
  if (B == 0) return 0;
  HcaParams p{};
  p.levels = levels;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.sink = sink;
  p.window = static_cast<const __nv_bfloat16*>(window);
  p.window_len = window_len;
  p.kv_pages = kv_pages;
  p.page_table = page_table;
  p.nblocks = nblocks;
  p.diag_kv = diag_kv;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.dbg = g_cta_debug;
  p.err = err;
  p.table_stride = table_stride;
  p.num_pages = num_pages;
  p.H = H;
  p.W = W;
  p.softmax_scale = softmax_scale;
  const int smem = bits == 4 ? HCfg<4>::SMEM : HCfg<8>::SMEM;
  auto kern = bits == 4 ? hca_attend_kernel<4> : hca_attend_kernel<8>;
  if (int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), smem, "hca decode")) return rc;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = kHcaCS;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t c = {};
  c.gridDim = dim3(B * kHcaCS);
  c.blockDim = dim3(kQThreads);
  c.dynamicSmemBytes = smem;
  c.stream = static_cast<cudaStream_t>(stream);
  c.attrs = at;
  c.numAttrs = pdl ? 2 : 1;
  AETHER_CUDA_TRY(cudaLaunchKernelEx(&c, kern, p), "hca decode: launch");
  return check_launch("hca_decode_paged");
}

int csa_decode_cta(const void* q, const float* index_q, const float* index_w, const float* sink, const void* window,
                   const int32_t* window_len, const uint8_t* idx_pages, const uint8_t* kv_pages,
                   const int32_t* page_table, int table_stride, int num_pages, const int32_t* nblocks,
                   int max_nblocks, const float* diag_idx, const float* diag_kv, int B, int H, int W, int bits,
                   int top_k, float softmax_scale, void* out, int32_t* sel_out, float* score_out, int score_stride,
                   uint32_t* workspace, int* err, int pdl, void* stream, const int32_t* rope_pos,
                   const float* rope_inv_freq, int rope_dim, const uint32_t* step_flags, uint32_t step_seq,
                   const float* levels) {
  int rc = check_common(bits, H, W, top_k, max_nblocks, table_stride, num_pages);
  AETHER_REQUIRE(!rope_inv_freq || (rope_pos && rope_dim > 0 && rope_dim <= kHeadDim && rope_dim % 4 == 0),
                 "csa decode: output RoPE needs positions and rope_dim in (0, 128], a multiple of 4");
  if (rc) return rc;
  AETHER_REQUIRE(workspace != nullptr, "csa decode: workspace is required");
  AETHER_REQUIRE(!score_out || max_nblocks <= kMaxKeys, "csa decode: score output is limited to %d blocks", kMaxKeys);
  if (B == 0) return 0;
  QParams p = base_params(q, index_q, index_w, sink, window, window_len, idx_pages, kv_pages, page_table, table_stride,
                          num_pages, nblocks, max_nblocks, diag_idx, diag_kv, H, W, top_k, softmax_scale, err);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.sel_out = sel_out;
  p.score_out = score_out;
  p.score_stride = score_stride;
  p.rope_pos = rope_pos;
  p.rope_inv_freq = rope_inv_freq;
  p.rope_dim = rope_dim;
  p.step_flags = step_flags;
  p.step_seq = step_seq;
  p.levels = levels;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  rc = bits == 4 ? run_decode<4>(p, B, max_nblocks, pdl != 0, st, reinterpret_cast<uint8_t*>(workspace))
                 : run_decode<8>(p, B, max_nblocks, pdl != 0, st, reinterpret_cast<uint8_t*>(workspace));
  if (rc) return rc;
  return check_launch("csa_decode");
}

// ----------------------------------------------------------- LSE merge
// out[b,h,:] = sum_r e^{m_r - M} O_r / (sum_r e^{m_r - M} l_r + e^{sink_h - M}),
// M = max(max_r m_r, sink_h): partial attention over disjoint source sets
// combined exactly (the sink counted once).  One warp per (b, h).
__global__ void lse_merge_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                                 long long stride_o, long long stride_ml, const float* __restrict__ sink, int G,
                                 int B, int H, __nv_bfloat16* __restrict__ out) {
  // rank r's partials: part_o + r * stride_o [B][H][128], part_ml + r * stride_ml [B][H][2]
  const int lane = threadIdx.x & 31;
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (w >= B * H) return;
  const int h = w % H;
  float M = sink[h];
  for (int r = 0; r < G; ++r) M = fmaxf(M, part_ml[r * stride_ml + w * 2]);
  float L = __expf(sink[h] - M);
  float acc[4] = {0, 0, 0, 0};
  for (int r = 0; r < G; ++r) {
    const float m = part_ml[r * stride_ml + w * 2], l = part_ml[r * stride_ml + w * 2 + 1];
    const float a = m == -INFINITY ? 0.f : __expf(m - M);
    L += a * l;
    const float4 o = *reinterpret_cast<const float4*>(part_o + r * stride_o + static_cast<long long>(w) * kHeadDim +
                                                      lane * 4);
    acc[0] += a * o.x;
    acc[1] += a * o.y;
    acc[2] += a * o.z;
    acc[3] += a * o.w;
  }
  const float inv = 1.f / L;
  __nv_bfloat162 o01 = __floats2bfloat162_rn(acc[0] * inv, acc[1] * inv);
  __nv_bfloat162 o23 = __floats2bfloat162_rn(acc[2] * inv, acc[3] * inv);
  *reinterpret_cast<uint2*>(out + static_cast<long long>(w) * kHeadDim + lane * 4) =
      make_uint2(*reinterpret_cast<uint32_t*>(&o01), *reinterpret_cast<uint32_t*>(&o23));
}

}  // namespace aether

using namespace aether;

// Profiling aid: when buf is non-null, later CSA decode launches record
// per-CTA phase timestamps (SM clock64 cycles) of the attend kernel into
// buf[cta * 16 + phase] and of the score kernel into buf[65536 + cta * 8 +
// phase]; buf must hold 65536 + 8 * (score grid size) entries.
extern "C" void aether_csa_decode_set_debug_timer(long long* buf) { aether::g_cta_debug = buf; }

extern "C" size_t aether_csa_decode_workspace_bytes(int B, int max_nblocks) {
  return aether::workspace_bytes(B > 0 ? B : 0, max_nblocks);
}

extern "C" int aether_csa_decode_smem_bytes(int bits) {
  return bits == 4 ? aether::QCfg<4, aether::kAttendCluster>::SMEM : aether::QCfg<8, aether::kAttendCluster>::SMEM;
}

// Context-parallel step 1: score this device's blocks [id_base, id_base +
// nblocks[b]) of every sequence and keep the top_k of each 8192-block chunk.
// cand_keys / cand_ids: [B][chunks * top_k], chunks = ceil(max_nblocks / 8192);
// padding entries have key 0 and id -1.
extern "C" int aether_csa_local_candidates(const float* index_q, const float* index_w, const uint8_t* idx_pages,
                                           const int32_t* page_table, int table_stride, int num_pages,
                                           const int32_t* nblocks, int max_nblocks, const float* diag_idx, int B,
                                           int bits, int top_k, int id_base, uint32_t* cand_keys, int32_t* cand_ids,
                                           void* workspace, int* err, void* stream) {
  int rc = check_common(bits, 1, 0, top_k, max_nblocks, table_stride, num_pages);
  if (rc) return rc;
  AETHER_REQUIRE(workspace && cand_keys && cand_ids, "csa_local_candidates: null buffer");
  AETHER_REQUIRE((top_k & 3) == 0, "csa_local_candidates: top_k must be a multiple of 4, got %d", top_k);
  if (B == 0) return 0;
  QParams p = base_params(nullptr, index_q, index_w, nullptr, nullptr, nullptr, idx_pages, nullptr, page_table,
                          table_stride, num_pages, nblocks, max_nblocks, diag_idx, nullptr, 1, 0, top_k, 0.f, err);
  p.ws = static_cast<uint32_t*>(workspace);
  p.id_base = id_base;
  p.chunks = max(1, (max_nblocks + kMaxKeys - 1) / kMaxKeys);
  p.sel_keys_out = cand_keys;
  p.sel_ids_out = cand_ids;
  p.sel_stride = top_k;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (bits == 4) {
    rc = set_smem_attrs<4>();
    if (!rc) rc = launch_score<4>(p, B, max_nblocks, false, st);
    if (!rc) rc = launch_attend<4>(p, B, true, st);
  } else {
    rc = set_smem_attrs<8>();
    if (!rc) rc = launch_score<8>(p, B, max_nblocks, false, st);
    if (!rc) rc = launch_attend<8>(p, B, true, st);
  }
  if (rc) return rc;
  return check_launch("csa_local_candidates");
}

// Context-parallel step 2: exact top_k over a merged candidate list (keys and
// ascending global ids, [B][cand_stride], cand_n used per row), attention over
// the winners this device holds (ids in [id_base, id_base + nblocks[b])) plus
// its window rows (window_len may be 0).  With part_o / part_ml given the
// un-normalised partial (O [B][H][128], (max, sum) [B][H][2]) is written for
// aether_lse_merge; otherwise the final bf16 output.  sel_out (optional)
// receives the global winners [B][top_k] in ascending order.
extern "C" int aether_csa_attend_candidates(const void* q, const float* sink, const void* window,
                                            const int32_t* window_len, const uint8_t* kv_pages,
                                            const int32_t* page_table, int table_stride, int num_pages,
                                            const int32_t* nblocks, int max_nblocks, const float* diag_kv,
                                            const uint32_t* cand_keys, const int32_t* cand_ids, int cand_n,
                                            int cand_stride, int id_base, int B, int H, int W, int bits, int top_k,
                                            float softmax_scale, void* out, int32_t* sel_out, float* part_o,
                                            float* part_ml, int* err, void* stream) {
  int rc = check_common(bits, H, W, top_k, max_nblocks, table_stride, num_pages);
  if (rc) return rc;
  AETHER_REQUIRE(cand_keys && cand_ids, "csa_attend_candidates: null candidate list");
  AETHER_REQUIRE(cand_n >= 0 && cand_n <= kMaxKeys && cand_stride >= cand_n,
                 "csa_attend_candidates: candidate count %d must be in [0, %d]", cand_n, kMaxKeys);
  AETHER_REQUIRE((cand_stride & 3) == 0, "csa_attend_candidates: cand_stride must be a multiple of 4");
  AETHER_REQUIRE((part_o == nullptr) == (part_ml == nullptr), "part_o and part_ml go together");
  AETHER_REQUIRE(part_o || out, "csa_attend_candidates: no output");
  if (B == 0) return 0;
  QParams p = base_params(q, nullptr, nullptr, sink, window, window_len, nullptr, kv_pages, page_table, table_stride,
                          num_pages, nblocks, max_nblocks, nullptr, diag_kv, H, W, top_k, softmax_scale, err);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.sel_out = sel_out;
  p.cand_keys = cand_keys;
  p.cand_ids = cand_ids;
  p.cand_n = cand_n;
  p.cand_stride = cand_stride;
  p.id_base = id_base;
  p.part_o = part_o;
  p.part_ml = part_ml;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  rc = bits == 4 ? set_smem_attrs<4>() : set_smem_attrs<8>();
  if (!rc) rc = bits == 4 ? launch_attend<4>(p, B, false, st) : launch_attend<8>(p, B, false, st);
  if (rc) return rc;
  return check_launch("csa_attend_candidates");
}

// Combine G partial attention results (from aether_csa_attend_candidates on
// G devices, gathered as part_o [G][B][H][128], part_ml [G][B][H][2]) with the
// per-head sink into the bf16 output [B][H][128].
extern "C" int aether_lse_merge(const float* part_o, const float* part_ml, const float* sink, int G, int B, int H,
                                void* out, void* stream) {
  AETHER_REQUIRE(G >= 1 && B >= 0 && H >= 1, "lse_merge: bad sizes");
  if (B == 0) return 0;
  const int warps = B * H;
  const long long bh = static_cast<long long>(B) * H;
  lse_merge_kernel<<<(warps * 32 + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      part_o, part_ml, bh * kHeadDim, bh * 2, sink, G, B, H, static_cast<__nv_bfloat16*>(out));
  return check_launch("lse_merge");
}

// As aether_lse_merge with rank r's partials at part_o + r * stride_o and
// part_ml + r * stride_ml (float elements), e.g. rows of an all-gathered
// buffer that packs each rank's [B][H][128] O and [B][H][2] (max, sum).
extern "C" int aether_lse_merge_strided(const float* part_o, const float* part_ml, long long stride_o,
                                        long long stride_ml, const float* sink, int G, int B, int H, void* out,
                                        void* stream) {
  AETHER_REQUIRE(G >= 1 && B >= 0 && H >= 1, "lse_merge: bad sizes");
  AETHER_REQUIRE(stride_o % 4 == 0 && (reinterpret_cast<uintptr_t>(part_o) & 15) == 0,
                 "lse_merge_strided: part_o rows must be 16-byte aligned");
  if (B == 0) return 0;
  const int warps = B * H;
  lse_merge_kernel<<<(warps * 32 + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      part_o, part_ml, stride_o, stride_ml, sink, G, B, H, static_cast<__nv_bfloat16*>(out));
  return check_launch("lse_merge_strided");
}
