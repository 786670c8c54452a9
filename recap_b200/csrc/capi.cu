// extern "C" entry points of librecap_b200.so (declared in include/recap_b200.h).
// Each entry point checks its shapes, builds the TMA tensor maps it needs from the raw
// device pointers, and launches on the given stream.  No entry point synchronises or
// allocates device memory (recap_peer_alloc, the allocator of buffers shared between ranks,
// aside); scratch buffers are passed in by the caller.
#include <cudaTypedefs.h>

#include <mutex>

#include "../../include/recap_b200.h"
#include <cstring>

#include "kernels.h"

namespace recap {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

void load_encode() {
  cudaDriverEntryPointQueryResult q;
  void* fn = nullptr;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
}

}  // namespace

int make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  std::call_once(g_encode_once, load_encode);
  if (g_encode == nullptr) return kErrLaunch;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (cols * 2) % 16 != 0 || box_rows == 0 ||
      box_rows > 256)
    return kErrShape;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                        box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : kErrShape;
}

struct Geom {
  int S, S_pad, NB, nB, nB_pad, rows, dense_start;
};

static bool geom(int S, int n_video, Geom* g) {
  if (S <= 0 || n_video <= 0 || n_video > S) return false;
  g->S = S;
  g->NB = (S + 127) / 128;
  g->S_pad = g->NB * 128;
  g->nB = (n_video + 127) / 128;
  g->nB_pad = ((g->nB + 127) / 128) * 128;
  g->rows = (n_video / 128) * 128;
  const bool shared_boundary = (n_video % 128) != 0 && S > n_video;
  g->dense_start = shared_boundary ? g->nB - 1 : g->nB;
  return true;
}

static bool d_ok(int D) { return D == 64 || D == 128; }

}  // namespace recap

using namespace recap;

extern "C" {

int recap_abi_version(void) { return RECAP_B200_ABI_VERSION; }

}  // extern "C"

// Token shards of a sequence-parallel layer: rank q holds native tokens
// [q tokens_per_rank, (q + 1) tokens_per_rank) of every tensor at ptr[t][q].
struct RankSources {
  int n_ranks, tokens_per_rank;
  const void* const* ptr[3];
};

static int gather_impl(const void* q, const void* k, const void* v, const RankSources* ranks,
                       const int64_t* strides, int batch, int heads, int S, int D, int n_video,
                       const int32_t* src_row, void* q_reordered, void* k_reordered, void* v_transposed,
                       float* q_mean, float* k_mean, float* v_mean, void* k_mean_bf16, void* v_mean_t_bf16,
                       void* k_centred_t, const float* basis, int rank, float* variance, void* variance_bf16,
                       float* k_norm_max, float* k_mean_norm, void* stream) {
  Geom g;
  if (!geom(S, n_video, &g) || !d_ok(D) || batch <= 0 || heads <= 0 || strides == nullptr ||
      src_row == nullptr)
    return kErrShape;
  GatherArgs a{};
  a.batch = batch;
  a.heads = heads;
  a.S = S;
  a.S_pad = g.S_pad;
  a.D = D;
  a.n_video = n_video;
  a.nB = g.nB;
  a.nB_pad = g.nB_pad;
  const void* src[3] = {q, k, v};
  for (int t = 0; t < 3; ++t) {
    a.src[t] = static_cast<const __nv_bfloat16*>(src[t]);
    a.stride_b[t] = strides[3 * t];
    a.stride_h[t] = strides[3 * t + 1];
    a.stride_s[t] = strides[3 * t + 2];
    if (src[t] && ((reinterpret_cast<uintptr_t>(src[t]) & 15) || (a.stride_b[t] % 8) ||
                   (a.stride_h[t] % 8) || (a.stride_s[t] % 8)))
      return kErrShape;
  }
  a.src_row = src_row;
  a.qr = static_cast<__nv_bfloat16*>(q_reordered);
  a.kr = static_cast<__nv_bfloat16*>(k_reordered);
  a.vt = static_cast<__nv_bfloat16*>(v_transposed);
  a.mean[0] = q_mean;
  a.mean[1] = k_mean;
  a.mean[2] = v_mean;
  a.kmean_bf16 = static_cast<__nv_bfloat16*>(k_mean_bf16);
  a.vmean_t_bf16 = static_cast<__nv_bfloat16*>(v_mean_t_bf16);
  a.kct = static_cast<__nv_bfloat16*>(k_centred_t);
  a.basis = basis;
  a.rank = rank;
  a.k_norm_max = k_norm_max;
  a.k_mean_norm = k_mean_norm;
  a.variance = variance;
  a.variance_bf16 = static_cast<__nv_bfloat16*>(variance_bf16);
  if ((a.kct != nullptr || a.variance != nullptr) && k == nullptr) return kErrShape;
  if (ranks != nullptr) {
    if (ranks->n_ranks < 2 || ranks->n_ranks > kMaxRanks || ranks->tokens_per_rank <= 0 ||
        static_cast<int64_t>(ranks->n_ranks) * ranks->tokens_per_rank != S || batch != 1)
      return kErrShape;
    a.n_ranks = ranks->n_ranks;
    a.tokens_per_rank = ranks->tokens_per_rank;
    for (int t = 0; t < 3; ++t) {
      if (src[t] == nullptr) continue;
      if (ranks->ptr[t] == nullptr) return kErrShape;
      for (int r = 0; r < ranks->n_ranks; ++r) {
        const void* p = ranks->ptr[t][r];
        if (p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15)) return kErrShape;
        a.rank_src[r][t] = static_cast<const __nv_bfloat16*>(p);
      }
    }
  }
  return launch_gather(a, static_cast<cudaStream_t>(stream));
}

extern "C" {

int recap_layout_gather(const void* q, const void* k, const void* v, const int64_t* strides, int batch,
                        int heads, int S, int D, int n_video, const int32_t* src_row, void* q_reordered,
                        void* k_reordered, void* v_transposed, float* q_mean, float* k_mean, float* v_mean,
                        void* k_mean_bf16, void* v_mean_t_bf16, void* k_centred_t, const float* basis, int rank,
                        float* variance, void* variance_bf16, float* k_norm_max, float* k_mean_norm,
                        void* stream) {
  return gather_impl(q, k, v, nullptr, strides, batch, heads, S, D, n_video, src_row, q_reordered, k_reordered,
                     v_transposed, q_mean, k_mean, v_mean, k_mean_bf16, v_mean_t_bf16, k_centred_t, basis, rank,
                     variance, variance_bf16, k_norm_max, k_mean_norm, stream);
}

int recap_layout_gather_ranks(const void* const* q_ranks, const void* const* k_ranks, const void* const* v_ranks,
                              int n_ranks, int tokens_per_rank, const int64_t* strides, int heads, int S, int D,
                              int n_video, const int32_t* src_row, void* q_reordered, void* k_reordered,
                              void* v_transposed, float* q_mean, float* k_mean, float* v_mean, void* k_mean_bf16,
                              void* v_mean_t_bf16, void* k_centred_t, const float* basis, int rank, float* variance,
                              void* variance_bf16, float* k_norm_max, float* k_mean_norm, void* stream) {
  if (q_ranks == nullptr || k_ranks == nullptr || v_ranks == nullptr) return kErrShape;
  RankSources rs{n_ranks, tokens_per_rank, {q_ranks, k_ranks, v_ranks}};
  return gather_impl(q_ranks[0], k_ranks[0], v_ranks[0], &rs, strides, 1, heads, S, D, n_video, src_row,
                     q_reordered, k_reordered, v_transposed, q_mean, k_mean, v_mean, k_mean_bf16, v_mean_t_bf16,
                     k_centred_t, basis, rank, variance, variance_bf16, k_norm_max, k_mean_norm, stream);
}

int recap_gather_max_rank(void) { return gather_max_rank(); }

int64_t recap_cvk_workspace_floats(int banks, int D, int n_video) {
  return static_cast<int64_t>(banks) * cvk_chunks(n_video) * D * D;
}

int recap_value_key_covariance(const void* v_transposed, const void* k_centred_t, int banks, int S, int D,
                               int n_video, float* workspace, float* cvk, void* cvk_bf16, int* status,
                               void* stream) {
  Geom g;
  if (!geom(S, n_video, &g) || !d_ok(D) || banks <= 0 || workspace == nullptr || cvk == nullptr)
    return kErrShape;
  CvkLaunch L{};
  L.D = D;
  int rc = kOk;
  rc |= make_tmap_bf16(&L.tm_vt, v_transposed, static_cast<uint64_t>(banks) * D, g.S_pad, 128);
  rc |= make_tmap_bf16(&L.tm_kct, k_centred_t, static_cast<uint64_t>(banks) * D, g.S_pad, D);
  if (rc != kOk) return kErrShape;
  L.args.banks = banks;
  L.args.n_video = n_video;
  L.args.video_steps = (n_video + 63) / 64;
  L.args.partial = workspace;
  L.args.status = status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  rc = launch_cvk(L, s);
  if (rc != kOk) return rc;
  return launch_moments_reduce(workspace, banks, cvk_chunks(n_video), D, 1.f / static_cast<float>(n_video), cvk,
                               static_cast<__nv_bfloat16*>(cvk_bf16), s);
}

int recap_pool_select(const float* q_mean, const float* k_mean, int banks, int nB, int D, int keep,
                      float scale, int n_video, int block_size, uint8_t* partition, void* stream) {
  if (!d_ok(D) || banks <= 0 || nB <= 0 || keep <= 0 || block_size != 128) return kErrShape;
  SelectArgs a{banks, nB, D, keep, n_video, block_size, scale, q_mean, k_mean, partition};
  return launch_select(a, static_cast<cudaStream_t>(stream));
}

int recap_partition_overlap(const uint8_t* new_partition, const uint8_t* old_partition, int64_t n,
                            long long* out2, void* stream) {
  OverlapArgs a{n, new_partition, old_partition, out2};
  return launch_overlap(a, static_cast<cudaStream_t>(stream));
}

int recap_kernel_block_mask(const uint8_t* partition, int banks, int S, int n_video, uint8_t* mask,
                            void* stream) {
  Geom g;
  if (!geom(S, n_video, &g)) return kErrShape;
  KernelMaskArgs a{banks, g.nB, g.NB, g.dense_start, partition, mask};
  return launch_kernel_mask(a, static_cast<cudaStream_t>(stream));
}

int64_t recap_closure_workspace_floats(int banks, int D, int n_video) {
  return closure_workspace_floats(banks, D, (n_video + 127) / 128);
}

int recap_closure_stats(const void* k_reordered, const void* v_transposed, const float* k_mean, int banks,
                        int S, int D, int n_video, int rank, const float* basis, float* scatter, float* cvk,
                        void* cvk_bf16, float* variance, void* variance_bf16, float* workspace,
                        void* stream) {
  Geom g;
  if (!geom(S, n_video, &g) || !d_ok(D) || banks <= 0) return kErrShape;
  ClosureArgs a{};
  a.banks = banks;
  a.S_pad = g.S_pad;
  a.D = D;
  a.n_video = n_video;
  a.nB = g.nB;
  a.nB_pad = g.nB_pad;
  a.rank = rank;
  a.kr = static_cast<const __nv_bfloat16*>(k_reordered);
  a.vt = static_cast<const __nv_bfloat16*>(v_transposed);
  a.kmean = k_mean;
  a.basis = basis;
  a.scatter = scatter;
  a.cvk = cvk;
  a.cvk_bf16 = static_cast<__nv_bfloat16*>(cvk_bf16);
  a.variance = variance;
  a.variance_bf16 = static_cast<__nv_bfloat16*>(variance_bf16);
  a.workspace = workspace;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((scatter || cvk) && workspace == nullptr) return kErrShape;
  int rc = launch_closure_moments(a, s);
  if (rc != kOk) return rc;
  if (basis != nullptr && variance != nullptr) rc = launch_closure_variance(a, s);
  return rc;
}

int recap_basis_prep(const float* basis, int banks, int D, void* basis_t_bf16, void* stream) {
  if (!d_ok(D) || banks <= 0) return kErrShape;
  BasisPrepArgs a{banks, D, basis, static_cast<__nv_bfloat16*>(basis_t_bf16)};
  return launch_basis_prep(a, static_cast<cudaStream_t>(stream));
}

int recap_coarse_tail(const void* q_reordered, const void* basis_t_bf16, const void* cvk_bf16,
                      const void* k_mean_bf16, const void* variance_bf16, const void* v_mean_t_bf16,
                      const uint8_t* partition, const float* counts_log, const float* k_mean_norm,
                      const float* old_lse, int banks, int S, int D, int n_video, float scale, float theta,
                      int rank, void* out, float* lse,
                      float* center_partial, float* center, int* status, void* stream) {
  Geom g;
  if (!geom(S, n_video, &g) || !d_ok(D) || banks <= 0) return kErrShape;
  if (old_lse != nullptr && (center_partial == nullptr || center == nullptr)) return kErrShape;
  CoarseLaunch L{};
  L.D = D;
  int rc = kOk;
  rc |= make_tmap_bf16(&L.tm_q, q_reordered, static_cast<uint64_t>(banks) * g.S_pad, D, 128);
  rc |= make_tmap_bf16(&L.tm_basis_t, basis_t_bf16, static_cast<uint64_t>(banks) * D, D, D);
  rc |= make_tmap_bf16(&L.tm_cvk, cvk_bf16, static_cast<uint64_t>(banks) * D, D, D);
  rc |= make_tmap_bf16(&L.tm_kmean, k_mean_bf16, static_cast<uint64_t>(banks) * g.nB_pad, D, 128);
  rc |= make_tmap_bf16(&L.tm_var, variance_bf16, static_cast<uint64_t>(banks) * g.nB_pad, D, 128);
  rc |= make_tmap_bf16(&L.tm_vmean_t, v_mean_t_bf16, static_cast<uint64_t>(banks) * D, g.nB_pad, D);
  if (rc != kOk) return kErrShape;
  CoarseArgs& a = L.args;
  a.banks = banks;
  a.S_pad = g.S_pad;
  a.D = D;
  a.nB = g.nB;
  a.nB_pad = g.nB_pad;
  a.rows = g.rows;
  a.n_video = n_video;
  a.scale = scale;
  a.theta = theta;
  a.rank = rank < 0 || rank >= D ? 0 : rank;
  a.partition = partition;
  a.k_mean_norm = k_mean_norm;
  a.counts_log = counts_log;
  a.old_lse = old_lse;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.lse = lse;
  a.center_partial = old_lse ? center_partial : nullptr;
  a.status = status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  rc = launch_coarse(L, s);
  if (rc != kOk || old_lse == nullptr) return rc;
  CenterArgs c{banks, g.rows / 128, g.rows, center_partial, center};
  return launch_center(c, s);
}

// Streaming multiprocessors of the current device (cached per device ordinal).
static int device_sm_count() {
  static int counts[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 1;
  if (dev >= 64) {
    int n = 1;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 1;
  }
  if (counts[dev] == 0) {
    int n = 1;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 1;
    counts[dev] = n;
  }
  return counts[dev];
}

// Output rows placed in the token shards of the ranks of a sequence-parallel layer.
struct OutRanks {
  void* const* ptr;
  int n_ranks, tokens_per_rank;
  int64_t bank_stride, row_stride;
};

static int apply_out_ranks(FmhaArgs& a, const OutRanks& o, int D) {
  if (o.ptr == nullptr || o.n_ranks < 2 || o.n_ranks > kMaxRanks || o.tokens_per_rank <= 0 ||
      static_cast<int64_t>(o.n_ranks) * o.tokens_per_rank != a.S || o.bank_stride % 8 || o.row_stride % 8 ||
      o.bank_stride < 0 || o.row_stride < D)
    return kErrShape;
  for (int r = 0; r < o.n_ranks; ++r) {
    if (o.ptr[r] == nullptr || (reinterpret_cast<uintptr_t>(o.ptr[r]) & 15)) return kErrShape;
    a.o_rank[r] = static_cast<__nv_bfloat16*>(o.ptr[r]);
  }
  a.o = a.o_rank[0];
  a.n_ranks = o.n_ranks;
  a.tokens_per_rank = o.tokens_per_rank;
  a.o_bank_stride = o.bank_stride;
  a.o_row_stride = o.row_stride;
  return kOk;
}

static int fmha_common(const void* q_reordered, const void* k_reordered, const void* v_transposed, int banks,
                       int S, int D, FmhaLaunch* L) {
  Geom g;
  (void)g;
  int rc = kOk;
  const int S_pad = ((S + 127) / 128) * 128;
  L->args.q = static_cast<const __nv_bfloat16*>(q_reordered);
  L->args.num_sms = device_sm_count();
  L->args.o_bank_stride = static_cast<int64_t>(S) * D;  // [banks, S, D] unless a caller places rows
  L->args.o_row_stride = D;
  rc |= make_tmap_bf16(&L->tm_q, q_reordered, static_cast<uint64_t>(banks) * S_pad, D, 128);
  rc |= make_tmap_bf16(&L->tm_k, k_reordered, static_cast<uint64_t>(banks) * S_pad, D, 128);
  rc |= make_tmap_bf16(&L->tm_vt, v_transposed, static_cast<uint64_t>(banks) * D, S_pad, D);
  return rc == kOk ? kOk : kErrShape;
}

int recap_block_sparse_fmha(const void* q_reordered, const void* k_reordered, const void* v_transposed,
                            const uint8_t* partition, const float* k_norm_max, int banks, int S, int D,
                            int n_video, int all_blocks, float scale, const int32_t* out_pos, void* out,
                            float* lse, int* status, void* stream) {
  Geom g;
  if (!geom(S, n_video, &g) || !d_ok(D) || banks <= 0 || out == nullptr) return kErrShape;
  if (!all_blocks && partition == nullptr) return kErrShape;
  FmhaLaunch L{};
  L.D = D;
  int rc = fmha_common(q_reordered, k_reordered, v_transposed, banks, S, D, &L);
  if (rc != kOk) return rc;
  FmhaArgs& a = L.args;
  a.banks = banks;
  a.S = S;
  a.S_pad = g.S_pad;
  a.NB = g.NB;
  a.nB = g.nB;
  a.dense_start = g.dense_start;
  a.rows = g.rows;
  a.all_blocks = all_blocks;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.partition = partition;
  a.k_norm_max = k_norm_max;
  a.epilogue = 0;
  a.out_pos = out_pos;
  a.o = static_cast<__nv_bfloat16*>(out);
  a.lse = lse;
  a.status = status;
  return launch_fmha(L, static_cast<cudaStream_t>(stream));
}

static int refresh_attention_impl(const void* q_reordered, const void* k_reordered, const void* v_transposed,
                                  const uint8_t* partition, const float* k_norm_max, int banks, int S, int D,
                                  int n_video, float scale, const int32_t* out_pos, void* out, float* lse,
                                  void* head_out, float* head_lse, int* status, void* stream,
                                  const OutRanks* sink) {
  Geom g;
  if (sink != nullptr && sink->ptr != nullptr) out = sink->ptr[0];
  if (!geom(S, n_video, &g) || !d_ok(D) || banks <= 0 || out == nullptr || lse == nullptr ||
      partition == nullptr || head_out == nullptr || head_lse == nullptr)
    return kErrShape;
  FmhaLaunch L{};
  L.D = D;
  int rc = fmha_common(q_reordered, k_reordered, v_transposed, banks, S, D, &L);
  if (rc != kOk) return rc;
  FmhaArgs& a = L.args;
  a.banks = banks;
  a.S = S;
  a.S_pad = g.S_pad;
  a.NB = g.NB;
  a.nB = g.nB;
  a.dense_start = g.dense_start;
  a.rows = g.rows;
  a.all_blocks = 1;
  a.refresh = 1;
  a.head_o = static_cast<__nv_bfloat16*>(head_out);
  a.head_lse = head_lse;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.partition = partition;
  a.k_norm_max = k_norm_max;
  a.epilogue = 0;
  a.out_pos = out_pos;
  a.o = static_cast<__nv_bfloat16*>(out);
  a.lse = lse;
  a.status = status;
  if (sink != nullptr && (rc = apply_out_ranks(a, *sink, D)) != kOk) return rc;
  return launch_fmha(L, static_cast<cudaStream_t>(stream));
}

int recap_refresh_attention(const void* q_reordered, const void* k_reordered, const void* v_transposed,
                            const uint8_t* partition, const float* k_norm_max, int banks, int S, int D,
                            int n_video, float scale, const int32_t* out_pos, void* out, float* lse,
                            void* head_out, float* head_lse, int* status, void* stream) {
  return refresh_attention_impl(q_reordered, k_reordered, v_transposed, partition, k_norm_max, banks, S, D, n_video,
                                scale, out_pos, out, lse, head_out, head_lse, status, stream, nullptr);
}

int recap_refresh_attention_ranks(const void* q_reordered, const void* k_reordered, const void* v_transposed,
                                  const uint8_t* partition, const float* k_norm_max, int banks, int S, int D,
                                  int n_video, float scale, const int32_t* out_pos, void* const* out_ranks,
                                  int n_ranks, int tokens_per_rank, int64_t out_bank_stride, int64_t out_row_stride,
                                  float* lse, void* head_out, float* head_lse, int* status, void* stream) {
  const OutRanks sink{out_ranks, n_ranks, tokens_per_rank, out_bank_stride, out_row_stride};
  if (out_ranks == nullptr) return kErrShape;
  return refresh_attention_impl(q_reordered, k_reordered, v_transposed, partition, k_norm_max, banks, S, D, n_video,
                                scale, out_pos, nullptr, lse, head_out, head_lse, status, stream, &sink);
}

static int sparse_step_impl(const void* q_reordered, const void* k_reordered, const void* v_transposed,
                            const uint8_t* partition, const float* k_norm_max, int banks, int S, int D, int n_video,
                            float scale, const void* coarse_out, const float* coarse_lse, const void* detail_value,
                            const float* detail_log_mass, const float* old_lse, const float* center,
                            const int32_t* out_pos, void* out, int* status, void* stream, const OutRanks* sink) {
  Geom g;
  if (sink != nullptr && sink->ptr != nullptr) out = sink->ptr[0];
  if (!geom(S, n_video, &g) || !d_ok(D) || banks <= 0 || out == nullptr || partition == nullptr) return kErrShape;
  if (g.rows > 0 && (coarse_out == nullptr || coarse_lse == nullptr || detail_value == nullptr ||
                     detail_log_mass == nullptr || old_lse == nullptr || center == nullptr))
    return kErrShape;
  FmhaLaunch L{};
  L.D = D;
  int rc = fmha_common(q_reordered, k_reordered, v_transposed, banks, S, D, &L);
  if (rc != kOk) return rc;
  FmhaArgs& a = L.args;
  a.banks = banks;
  a.S = S;
  a.S_pad = g.S_pad;
  a.NB = g.NB;
  a.nB = g.nB;
  a.dense_start = g.dense_start;
  a.rows = g.rows;
  a.all_blocks = 0;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.partition = partition;
  a.k_norm_max = k_norm_max;
  a.epilogue = 1;
  a.out_pos = out_pos;
  a.o = static_cast<__nv_bfloat16*>(out);
  a.lse = nullptr;
  a.go = static_cast<const __nv_bfloat16*>(coarse_out);
  a.gl = coarse_lse;
  a.det = static_cast<const __half*>(detail_value);
  a.dl = detail_log_mass;
  a.ogl = old_lse;
  a.center = center;
  a.status = status;
  a.tma_epilogue = 0;
  if (g.rows > 0) {
    // the epilogue stages each tile's coarse output and refinement through shared memory
    // (both 2-byte elements: the copies move bytes)
    const uint64_t vrows = static_cast<uint64_t>(banks) * g.rows;
    rc = make_tmap_bf16(&L.tm_go, coarse_out, vrows, D, 128);
    if (rc == kOk) rc = make_tmap_bf16(&L.tm_det, detail_value, vrows, D, 128);
    if (rc != kOk) return rc;
    a.tma_epilogue = 1;
  }
  if (sink != nullptr && (rc = apply_out_ranks(a, *sink, D)) != kOk) return rc;
  return launch_fmha(L, static_cast<cudaStream_t>(stream));
}

int recap_sparse_step(const void* q_reordered, const void* k_reordered, const void* v_transposed,
                      const uint8_t* partition, const float* k_norm_max, int banks, int S, int D, int n_video,
                      float scale,
                      const void* coarse_out, const float* coarse_lse, const void* detail_value,
                      const float* detail_log_mass, const float* old_lse, const float* center,
                      const int32_t* out_pos, void* out, int* status, void* stream) {
  return sparse_step_impl(q_reordered, k_reordered, v_transposed, partition, k_norm_max, banks, S, D, n_video, scale,
                          coarse_out, coarse_lse, detail_value, detail_log_mass, old_lse, center, out_pos, out,
                          status, stream, nullptr);
}

int recap_sparse_step_ranks(const void* q_reordered, const void* k_reordered, const void* v_transposed,
                            const uint8_t* partition, const float* k_norm_max, int banks, int S, int D, int n_video,
                            float scale, const void* coarse_out, const float* coarse_lse, const void* detail_value,
                            const float* detail_log_mass, const float* old_lse, const float* center,
                            const int32_t* out_pos, void* const* out_ranks, int n_ranks, int tokens_per_rank,
                            int64_t out_bank_stride, int64_t out_row_stride, int* status, void* stream) {
  const OutRanks sink{out_ranks, n_ranks, tokens_per_rank, out_bank_stride, out_row_stride};
  if (out_ranks == nullptr) return kErrShape;
  return sparse_step_impl(q_reordered, k_reordered, v_transposed, partition, k_norm_max, banks, S, D, n_video, scale,
                          coarse_out, coarse_lse, detail_value, detail_log_mass, old_lse, center, out_pos, nullptr,
                          status, stream, &sink);
}

int recap_exp2_check(const float* in, float* out, int n, void* stream) {
  return launch_exp2_check(in, out, n, static_cast<cudaStream_t>(stream));
}

int recap_wait_selftest(int* status, long long limit_ns, long long* result, void* stream) {
  return launch_wait_selftest(status, limit_ns, result, static_cast<cudaStream_t>(stream));
}

int recap_refresh_partials(int banks, int n_video) {
  return refresh_partials_count(banks, (n_video / 128) * 128);
}

int recap_refresh_detail(const void* full_o, const float* full_lse, const void* head_o, const float* head_lse,
                         const void* coarse_out, const float* coarse_lse, const int32_t* perm, int banks, int S,
                         int D, int n_video, int video_offset, void* detail_value, float* detail_log_mass,
                         int validate, const float* old_lse, const float* center, float* partials,
                         float* stats, void* stream) {
  Geom g;
  if (!geom(S, n_video, &g) || !d_ok(D) || banks <= 0) return kErrShape;
  if (validate && (partials == nullptr || stats == nullptr)) return kErrShape;
  if ((old_lse == nullptr) != (center == nullptr)) return kErrShape;
  if (old_lse != nullptr && !validate) return kErrShape;  // the drift weight only affects validation
  RefreshArgs a{};
  a.banks = banks;
  a.S = S;
  a.D = D;
  a.rows = g.rows;
  a.video_offset = video_offset;
  a.full_o = static_cast<const __nv_bfloat16*>(full_o);
  a.full_lse = full_lse;
  a.head_o = static_cast<const __nv_bfloat16*>(head_o);
  a.head_lse = head_lse;
  a.go = static_cast<const __nv_bfloat16*>(coarse_out);
  a.gl = coarse_lse;
  a.perm = perm;
  a.det = static_cast<__half*>(detail_value);
  a.dl = detail_log_mass;
  a.validate = validate;
  a.ogl = old_lse;
  a.center = center;
  a.partials = partials;
  a.stats = stats;
  return launch_refresh(a, static_cast<cudaStream_t>(stream));
}

int recap_refresh_detail_noalloc(const void* full_o, const float* full_lse, const void* head_o,
                                 const float* head_lse, const void* coarse_out, const float* coarse_lse,
                                 const int32_t* perm, int banks, int S, int D, int n_video, int video_offset,
                                 void* detail_value, float* detail_log_mass, int validate, const float* old_lse,
                                 const float* center, float* stats, void* stream) {
  Geom g;
  if (!geom(S, n_video, &g) || !d_ok(D) || banks <= 0) return kErrShape;
  if (validate && stats == nullptr) return kErrShape;
  if ((old_lse == nullptr) != (center == nullptr)) return kErrShape;
  if (old_lse != nullptr && !validate) return kErrShape;
  RefreshArgs a{};
  a.banks = banks;
  a.S = S;
  a.D = D;
  a.rows = g.rows;
  a.video_offset = video_offset;
  a.full_o = static_cast<const __nv_bfloat16*>(full_o);
  a.full_lse = full_lse;
  a.head_o = static_cast<const __nv_bfloat16*>(head_o);
  a.head_lse = head_lse;
  a.go = static_cast<const __nv_bfloat16*>(coarse_out);
  a.gl = coarse_lse;
  a.perm = perm;
  a.det = static_cast<__half*>(detail_value);
  a.dl = detail_log_mass;
  a.validate = validate;
  a.ogl = old_lse;
  a.center = center;
  a.partials = nullptr;
  a.stats = stats;
  return launch_refresh_noalloc(a, static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------- buffers shared between ranks

int recap_peer_alloc(int64_t bytes, void** ptr) {
  if (bytes <= 0 || ptr == nullptr) return kErrShape;
  return cudaMalloc(ptr, static_cast<size_t>(bytes)) == cudaSuccess ? kOk : kErrLaunch;
}

int recap_peer_free(void* ptr) { return cudaFree(ptr) == cudaSuccess ? kOk : kErrLaunch; }

int recap_peer_handle_bytes(void) { return static_cast<int>(sizeof(cudaIpcMemHandle_t)); }

int recap_peer_export(void* ptr, void* handle_out) {
  if (ptr == nullptr || handle_out == nullptr) return kErrShape;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return kErrLaunch;
  std::memcpy(handle_out, &h, sizeof(h));
  return kOk;
}

int recap_peer_import(const void* handle, void** ptr) {
  if (handle == nullptr || ptr == nullptr) return kErrShape;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? kOk : kErrLaunch;
}

int recap_peer_close(void* ptr) { return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? kOk : kErrLaunch; }

int recap_push_heads(const void* src, int tokens, int heads, int D, int rank, int n_ranks,
                     void* const* recv_ranks, void* stream) {
  if (src == nullptr || recv_ranks == nullptr || tokens <= 0 || (D != 64 && D != 128) || n_ranks < 1 ||
      n_ranks > kMaxRanks || heads <= 0 || heads % n_ranks || rank < 0 || rank >= n_ranks ||
      (reinterpret_cast<uintptr_t>(src) & 15))
    return kErrShape;
  PushArgs a{};
  a.tokens = tokens;
  a.heads = heads;
  a.heads_per_rank = heads / n_ranks;
  a.D = D;
  a.token0 = static_cast<int64_t>(rank) * tokens;
  a.src = static_cast<const __nv_bfloat16*>(src);
  for (int q = 0; q < n_ranks; ++q) {
    if (recv_ranks[q] == nullptr || (reinterpret_cast<uintptr_t>(recv_ranks[q]) & 15)) return kErrShape;
    a.dst[q] = static_cast<__nv_bfloat16*>(recv_ranks[q]);
  }
  return launch_push(a, static_cast<cudaStream_t>(stream));
}

int recap_scatter_rows(const void* src, int banks, int S, int D, void* const* out_ranks, int n_ranks,
                       int tokens_per_rank, int64_t out_bank_stride, int64_t out_row_stride, void* stream) {
  if (src == nullptr || out_ranks == nullptr || banks <= 0 || S <= 0 || (D != 64 && D != 128) ||
      n_ranks < 1 || n_ranks > kMaxRanks || tokens_per_rank <= 0 ||
      static_cast<int64_t>(n_ranks) * tokens_per_rank != S || out_bank_stride < 0 || out_row_stride < D ||
      out_bank_stride % 8 || out_row_stride % 8 || (reinterpret_cast<uintptr_t>(src) & 15))
    return kErrShape;
  ScatterArgs a{};
  a.banks = banks;
  a.S = S;
  a.D = D;
  a.tokens_per_rank = tokens_per_rank;
  a.bank_stride = out_bank_stride;
  a.row_stride = out_row_stride;
  a.src = static_cast<const __nv_bfloat16*>(src);
  for (int q = 0; q < n_ranks; ++q) {
    if (out_ranks[q] == nullptr || (reinterpret_cast<uintptr_t>(out_ranks[q]) & 15)) return kErrShape;
    a.dst[q] = static_cast<__nv_bfloat16*>(out_ranks[q]);
  }
  return launch_scatter(a, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
