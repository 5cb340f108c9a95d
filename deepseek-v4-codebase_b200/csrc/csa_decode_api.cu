// C-ABI entry points of the fused paged decode (sm_100a): CSA and HCA decode
// steps, the fused inverse-RoPE and score-output variants, and the
// host-buffer forms (one call per step, or a prepared plan) that copy a
// step's packed inputs from pinned host memory, run the decode and copy the
// results back.  The kernels are in csa_decode_cta.cu.
//
// Reference data flow replaced: aether_2b/serving.py:597-625 (CSA) and
// :507-522 (HCA) plus the attention backend call at :450-467.
#include "aether_b200.h"
#include "capi_util.cuh"
#include "common.cuh"

namespace aether {

int hca_decode_cta(const void* q, const float* sink, const void* window, const int32_t* window_len,
                   const uint8_t* kv_pages, const int32_t* page_table, int table_stride, int num_pages,
                   const int32_t* nblocks, int max_nblocks, const float* diag_kv, int B, int H, int W, int bits,
                   float softmax_scale, void* out, int* err, int pdl, void* stream, const float* levels = nullptr);
int csa_decode_cta(const void* q, const float* index_q, const float* index_w, const float* sink, const void* window,
                   const int32_t* window_len, const uint8_t* idx_pages, const uint8_t* kv_pages,
                   const int32_t* page_table, int table_stride, int num_pages, const int32_t* nblocks,
                   int max_nblocks, const float* diag_idx, const float* diag_kv, int B, int H, int W, int bits,
                   int top_k, float softmax_scale, void* out, int32_t* sel_out, float* score_out, int score_stride,
                   uint32_t* workspace, int* err, int pdl, void* stream,
                   const int32_t* rope_pos = nullptr, const float* rope_inv_freq = nullptr,
                   int rope_dim = 0, const uint32_t* step_flags = nullptr, uint32_t step_seq = 0,
                   const float* levels = nullptr);

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
  AETHER_REQUIRE(cluster <= 1, "csa_decode_paged: cluster must be 0 (the per-sequence cluster kernels were removed)");
  return csa_decode_cta(q, index_q, index_w, sink, window, window_len, idx_pages, kv_pages, page_table,
                        table_stride, num_pages, nblocks, max_nblocks, diag_idx, diag_kv, B, H, W, bits, top_k,
                        softmax_scale, out, sel_out, nullptr, 0, workspace, err, pdl, stream);
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
  AETHER_REQUIRE(cluster <= 0, "hca_decode_paged: cluster must be 0 (the per-sequence cluster kernels were removed)");
  return hca_decode_cta(q, sink, window, window_len, kv_pages, page_table, table_stride, num_pages, nblocks,
                        max_nblocks, diag_kv, B, H, W, bits, softmax_scale, out, err, pdl, stream);
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
  AETHER_REQUIRE(cluster <= 1, "csa_decode_paged: cluster must be 0 (the per-sequence cluster kernels were removed)");
  return csa_decode_cta(q, index_q, index_w, sink, window, window_len, idx_pages, kv_pages, page_table, table_stride,
                        num_pages, nblocks, max_nblocks, diag_idx, diag_kv, B, H, W, bits, top_k, softmax_scale, out,
                        sel_out, score_out, score_stride, workspace, err, pdl, stream);
}


// aether_csa_decode_paged for a cache in the Lloyd-Max level format: codes
// are indices into levels [2^bits] (fp32), entries levels[c] * scale in the
// rotated domain.  The level table is applied inside the score and attend
// kernels (no dequantized copy of the cache).
int aether_csa_decode_paged_levels(const void* q, const float* index_q, const float* index_w, const float* sink,
                                   const void* window, const int32_t* window_len, const uint8_t* idx_pages,
                                   const uint8_t* kv_pages, const int32_t* page_table, int table_stride,
                                   int num_pages, const int32_t* nblocks, int max_nblocks, const float* diag_idx,
                                   const float* diag_kv, int B, int H, int W, int bits, int top_k,
                                   float softmax_scale, const float* levels, void* out, int32_t* sel_out,
                                   uint32_t* workspace, int* err, int pdl, void* stream) {
  AETHER_REQUIRE(index_q && index_w && idx_pages && diag_idx, "csa_decode_paged: null index input");
  AETHER_REQUIRE(levels, "csa_decode_paged_levels: null level table");
  return csa_decode_cta(q, index_q, index_w, sink, window, window_len, idx_pages, kv_pages, page_table,
                        table_stride, num_pages, nblocks, max_nblocks, diag_idx, diag_kv, B, H, W, bits, top_k,
                        softmax_scale, out, sel_out, nullptr, 0, workspace, err, pdl, stream, nullptr, nullptr, 0,
                        nullptr, 0, levels);
}

// aether_hca_decode_paged for a cache in the Lloyd-Max level format.
int aether_hca_decode_paged_levels(const void* q, const float* sink, const void* window, const int32_t* window_len,
                                   const uint8_t* kv_pages, const int32_t* page_table, int table_stride,
                                   int num_pages, const int32_t* nblocks, int max_nblocks, const float* diag_kv,
                                   int B, int H, int W, int bits, float softmax_scale, const float* levels,
                                   void* out, int* err, int pdl, void* stream) {
  AETHER_REQUIRE(levels, "hca_decode_paged_levels: null level table");
  return hca_decode_cta(q, sink, window, window_len, kv_pages, page_table, table_stride, num_pages, nblocks,
                        max_nblocks, diag_kv, B, H, W, bits, softmax_scale, out, err, pdl, stream, levels);
}

}  // extern "C"
