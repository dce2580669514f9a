// Python bindings of the wavelet_b200 CUDA extension.  Thin torch::Tensor
// wrappers that check dtypes/shapes/strides and forward raw pointers plus the
// current CUDA stream to the kernel launchers.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "attention.h"
#include "comm.h"
#include "moe.h"
#include "policy.h"
#include "decode.h"
#include "gemm.h"
#include "kernels.h"

namespace wb {
int* error_word(int device);
int read_error_word(int device);
long long launch_count();
void note_launches(long long n);
void clear_error_word(int device);
}  // namespace wb

namespace {

#define WB_CHECK(cond, msg) TORCH_CHECK(cond, "wavelet_b200: ", msg)

inline cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

inline void check_cuda(const at::Tensor& t, const char* name) {
  WB_CHECK(t.is_cuda(), std::string(name) + " must be a CUDA tensor");
}
inline void check_bf16(const at::Tensor& t, const char* name) {
  check_cuda(t, name);
  WB_CHECK(t.scalar_type() == at::kBFloat16, std::string(name) + " must be bfloat16");
}
inline void check_f32(const at::Tensor& t, const char* name) {
  check_cuda(t, name);
  WB_CHECK(t.scalar_type() == at::kFloat, std::string(name) + " must be float32");
}

// Leading dimension of a 2-D view whose inner stride is 1.
inline int64_t ld_of(const at::Tensor& t, const char* name) {
  WB_CHECK(t.dim() == 2, std::string(name) + " must be 2-D");
  WB_CHECK(t.stride(1) == 1 || t.size(1) == 1, std::string(name) + " inner stride must be 1");
  return t.size(0) == 1 ? std::max<int64_t>(t.stride(0), t.size(1)) : t.stride(0);
}

// C[M,N] (op)= alpha * A(m,k) B(n,k) (+bias).
//   a: [M,K] (a_mn=false) or [K,M] (a_mn=true);  b: [N,K] or [K,N].
void gemm(const at::Tensor& a, bool a_mn, const at::Tensor& b, bool b_mn, at::Tensor& c,
          int64_t epi, double alpha, const c10::optional<at::Tensor>& bias,
          const c10::optional<at::Tensor>& res) {
  check_bf16(a, "a");
  check_bf16(b, "b");
  check_cuda(c, "c");
  const c10::cuda::CUDAGuard guard(a.device());
  wb::GemmArgs g;
  g.A = a.data_ptr();
  g.lda = ld_of(a, "a");
  g.a_mn = a_mn;
  g.B = b.data_ptr();
  g.ldb = ld_of(b, "b");
  g.b_mn = b_mn;
  g.M = a_mn ? a.size(1) : a.size(0);
  const int64_t ka = a_mn ? a.size(0) : a.size(1);
  g.N = b_mn ? b.size(1) : b.size(0);
  const int64_t kb = b_mn ? b.size(0) : b.size(1);
  WB_CHECK(ka == kb, "gemm: K mismatch");
  g.K = ka;
  WB_CHECK(c.dim() == 2 && c.size(0) == g.M && c.size(1) == g.N, "gemm: bad output shape");
  g.C = c.data_ptr();
  g.ldc = ld_of(c, "c");
  g.epi = static_cast<int>(epi);
  if (g.epi == wb::kEpiBF16)
    check_bf16(c, "c");
  else
    check_f32(c, "c");
  g.alpha = static_cast<float>(alpha);
  if (bias.has_value() && bias->defined()) {
    check_bf16(*bias, "bias");
    WB_CHECK(bias->numel() == g.N && bias->is_contiguous(), "gemm: bias must be [N]");
    WB_CHECK(g.epi == wb::kEpiBF16, "gemm: bias only with the bf16 epilogue");
    g.bias = bias->data_ptr();
  }
  if (res.has_value() && res->defined()) {
    check_bf16(*res, "res");
    WB_CHECK(res->dim() == 2 && res->size(0) == g.M && res->size(1) == g.N,
             "gemm: residual must be [M, N]");
    WB_CHECK(g.epi == wb::kEpiBF16, "gemm: residual only with the bf16 epilogue");
    g.res = res->data_ptr();
    g.ldr = ld_of(*res, "res");
  }
  wb::gemm_bf16(g, cur_stream());
}

// Extended GEMM: optional second operand pair (LoRA-fused linear) and/or an
// NF4 B operand (QLoRA base weight).  b is ignored when q is given.
void gemm_ex(const at::Tensor& a, bool a_mn, const c10::optional<at::Tensor>& b, bool b_mn, at::Tensor& c,
             int64_t N, int64_t epi, double alpha, const c10::optional<at::Tensor>& bias,
             const c10::optional<at::Tensor>& res, const c10::optional<at::Tensor>& a2,
             const c10::optional<at::Tensor>& b2, const c10::optional<at::Tensor>& q,
             const c10::optional<at::Tensor>& q_absmax, int64_t q_rows, int64_t q_cols,
             const std::vector<double>& lut) {
  check_bf16(a, "a");
  check_cuda(c, "c");
  const c10::cuda::CUDAGuard guard(a.device());
  wb::GemmArgs g;
  g.A = a.data_ptr();
  g.lda = ld_of(a, "a");
  g.a_mn = a_mn;
  g.b_mn = b_mn;
  g.M = a_mn ? a.size(1) : a.size(0);
  g.K = a_mn ? a.size(0) : a.size(1);
  g.N = N;
  if (q) {
    WB_CHECK(q->scalar_type() == at::kByte && q->is_cuda() && q->is_contiguous(), "gemm_ex: q must be contiguous uint8 CUDA");
    WB_CHECK(q_absmax && q_absmax->scalar_type() == at::kFloat && q_absmax->is_contiguous(), "gemm_ex: q_absmax fp32");
    WB_CHECK(lut.size() == 16, "gemm_ex: lut must have 16 entries");
    WB_CHECK(q->numel() == q_rows * q_cols / 2 && q_absmax->numel() == q_rows * q_cols / 64, "gemm_ex: NF4 sizes");
    WB_CHECK((reinterpret_cast<uintptr_t>(q->data_ptr()) & 15) == 0, "gemm_ex: q must be 16-byte aligned");
    g.q = q->data_ptr<uint8_t>();
    g.q_absmax = q_absmax->data_ptr<float>();
    g.q_rows = q_rows;
    g.q_cols = q_cols;
    for (int i = 0; i < 16; ++i) g.q_lut[i] = static_cast<float>(lut[i]);
  } else {
    WB_CHECK(b.has_value(), "gemm_ex: b or q required");
    check_bf16(*b, "b");
    g.B = b->data_ptr();
    g.ldb = ld_of(*b, "b");
  }
  if (a2) {
    WB_CHECK(b2.has_value(), "gemm_ex: a2 needs b2");
    check_bf16(*a2, "a2");
    check_bf16(*b2, "b2");
    g.A2 = a2->data_ptr();
    g.lda2 = ld_of(*a2, "a2");
    g.B2 = b2->data_ptr();
    g.ldb2 = ld_of(*b2, "b2");
    g.K2 = a_mn ? a2->size(0) : a2->size(1);
  }
  g.C = c.data_ptr();
  g.ldc = ld_of(c, "c");
  g.epi = static_cast<int>(epi);
  g.alpha = static_cast<float>(alpha);
  if (bias) {
    check_bf16(*bias, "bias");
    g.bias = bias->data_ptr();
  }
  if (res) {
    check_bf16(*res, "res");
    g.res = res->data_ptr();
    g.ldr = ld_of(*res, "res");
  }
  wb::gemm_bf16(g, cur_stream());
}

// Grouped (MoE expert) GEMM.  mode 1: C = A B_g^T with g = tile_group[m_tile];
// mode 2: C[g*M:(g+1)*M] (op)= A_g^T B_g over token segments (k_start, k_len).
void gemm_grouped(const at::Tensor& a, bool a_mn, const at::Tensor& b, bool b_mn, at::Tensor& c, int64_t mode,
                  int64_t M, int64_t N, int64_t K, const c10::optional<at::Tensor>& tile_group,
                  int64_t b_group_stride, int64_t b_outer, const c10::optional<at::Tensor>& k_start,
                  const c10::optional<at::Tensor>& k_len, int64_t groups, int64_t epi, double alpha) {
  check_bf16(a, "a");
  check_bf16(b, "b");
  check_cuda(c, "c");
  const c10::cuda::CUDAGuard guard(a.device());
  wb::GemmArgs g;
  g.A = a.data_ptr();
  g.lda = ld_of(a, "a");
  g.a_mn = a_mn;
  g.B = b.data_ptr();
  g.ldb = ld_of(b, "b");
  g.b_mn = b_mn;
  g.C = c.data_ptr();
  g.ldc = ld_of(c, "c");
  g.M = M;
  g.N = N;
  g.K = K;
  g.epi = static_cast<int>(epi);
  g.alpha = static_cast<float>(alpha);
  g.group_mode = static_cast<int>(mode);
  if (tile_group) {
    WB_CHECK(tile_group->scalar_type() == at::kInt && tile_group->is_cuda(), "gemm_grouped: tile_group int32 CUDA");
    g.tile_group = tile_group->data_ptr<int>();
  }
  g.b_group_stride = b_group_stride;
  g.b_outer = b_outer;
  if (k_start) g.k_start = k_start->data_ptr<int>();
  if (k_len) g.k_len = k_len->data_ptr<int>();
  g.groups = static_cast<int>(groups);
  wb::gemm_bf16(g, cur_stream());
}

// ------------------------------------------------------------ peer fabric
int64_t fabric_malloc_(int64_t nbytes, int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  return reinterpret_cast<int64_t>(wb::fabric_malloc(static_cast<size_t>(nbytes)));
}
void fabric_free_(int64_t p) { wb::fabric_free(reinterpret_cast<void*>(p)); }
py::bytes fabric_export_(int64_t p) {
  unsigned char h[64];
  wb::fabric_export(reinterpret_cast<void*>(p), h);
  return py::bytes(reinterpret_cast<const char*>(h), 64);
}
int64_t fabric_import_(const std::string& h, int64_t device) {
  WB_CHECK(h.size() == 64, "fabric_import: handle must be 64 bytes");
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  return reinterpret_cast<int64_t>(wb::fabric_import(reinterpret_cast<const unsigned char*>(h.data())));
}
void fabric_close_(int64_t p) { wb::fabric_close(reinterpret_cast<void*>(p)); }

// A tensor view of fabric memory (the fabric owns the allocation).
at::Tensor from_ptr(int64_t p, int64_t numel, at::ScalarType dtype, int64_t device) {
  auto opts = at::TensorOptions().dtype(dtype).device(at::kCUDA, static_cast<c10::DeviceIndex>(device));
  return at::from_blob(reinterpret_cast<void*>(p), {numel}, [](void*) {}, opts);
}

inline wb::PeerPtrs peers_of(const std::vector<int64_t>& v, int world) {
  WB_CHECK(world >= 1 && world <= wb::kMaxPeers && (int)v.size() >= world, "bad peer pointer list");
  wb::PeerPtrs pp{};
  for (int i = 0; i < world; ++i) pp.p[i] = reinterpret_cast<void*>(v[i]);
  return pp;
}

void peer_barrier(const std::vector<int64_t>& pads, int64_t rank, int64_t world, int64_t epoch, int64_t slot_base,
                  double budget_s) {
  int dev = 0;
  cudaGetDevice(&dev);
  wb::peer_barrier(peers_of(pads, (int)world), (int)rank, (int)world, static_cast<uint32_t>(epoch), (int)slot_base,
                   static_cast<uint64_t>(budget_s * 1e9), wb::error_word(dev), cur_stream());
}

void rs_sum_sumsq(const std::vector<int64_t>& grads, int64_t world, int64_t lo, int64_t n, double scale,
                  at::Tensor& out, at::Tensor& stats, int64_t w_end, double w_lo) {
  check_f32(out, "out");
  check_f32(stats, "stats");
  WB_CHECK(out.numel() >= n, "rs_sum_sumsq: out too small");
  wb::rs_sum_sumsq(peers_of(grads, (int)world), (int)world, lo, n, (float)scale, out.data_ptr<float>(),
                   stats.data_ptr<float>(), w_end, (float)w_lo, cur_stream());
}

void norm_exchange(const std::vector<int64_t>& pads, int64_t rank, int64_t world, int64_t epoch,
                   const at::Tensor& stats, double max_norm, at::Tensor& tot, double budget_s) {
  check_f32(stats, "stats");
  check_f32(tot, "tot");
  int dev = 0;
  cudaGetDevice(&dev);
  wb::norm_exchange(peers_of(pads, (int)world), (int)rank, (int)world, static_cast<uint32_t>(epoch),
                    stats.data_ptr<float>(), (float)max_norm, tot.data_ptr<float>(),
                    static_cast<uint64_t>(budget_s * 1e9), wb::error_word(dev), cur_stream());
}

void adamw_allgather(const std::vector<int64_t>& compute, int64_t world, int64_t lo, at::Tensor& master,
                     const at::Tensor& g, at::Tensor& m, at::Tensor& v, double lr, double b1, double b2, double eps,
                     double wd, int64_t step, const at::Tensor& tot) {
  check_f32(master, "master");
  check_f32(g, "g");
  check_f32(m, "m");
  check_f32(v, "v");
  check_f32(tot, "tot");
  const float bc1 = 1.f - std::pow((float)b1, (float)step);
  const float bc2 = 1.f - std::pow((float)b2, (float)step);
  wb::adamw_allgather(peers_of(compute, (int)world), (int)world, lo, master.data_ptr<float>(), g.data_ptr<float>(),
                      m.data_ptr<float>(), v.data_ptr<float>(), master.numel(), (float)lr, (float)b1, (float)b2,
                      (float)eps, (float)wd, bc1, bc2, tot.data_ptr<float>(), cur_stream());
}

void gather_from_peers(const std::vector<int64_t>& src, int64_t world, int64_t off, int64_t n, at::Tensor& dst) {
  check_bf16(dst, "dst");
  WB_CHECK(dst.is_contiguous() && dst.numel() >= n * world, "gather_from_peers: dst too small");
  wb::gather_from_peers(peers_of(src, (int)world), (int)world, off, n, dst.data_ptr(), cur_stream());
}

// Policy push: seg is a host int64 table [nseg, 6] (src_off, dst_off, rows,
// row_len, src_stride, dst_stride); every block is checked against the source
// tensor and dst_numel here, before anything is launched.  Returns the vector
// width used (8 / 4 when every term is aligned to it, else 1).
int64_t policy_push(const at::Tensor& src, const std::vector<int64_t>& dst, int64_t dst_numel, bool dst_bf16,
                    const at::Tensor& seg) {
  check_cuda(src, "src");
  WB_CHECK(src.is_contiguous() && (src.scalar_type() == at::kBFloat16 || src.scalar_type() == at::kFloat),
           "policy_push: src must be a contiguous bf16 / fp32 tensor");
  WB_CHECK(!seg.is_cuda() && seg.scalar_type() == at::kLong && seg.dim() == 2 && seg.size(1) == 6 && seg.is_contiguous(),
           "policy_push: seg must be a contiguous host int64 [nseg, 6] table");
  const int nd = (int)dst.size();
  WB_CHECK(nd >= 1 && nd <= wb::kMaxPeers, "policy_push: 1..8 destinations");
  const bool src_bf16 = src.scalar_type() == at::kBFloat16;
  const int64_t n = seg.size(0);
  if (n == 0) return 0;
  const int64_t* g = seg.data_ptr<int64_t>();
  const int want = (src_bf16 || dst_bf16) ? 8 : 4;  // 16-byte loads and stores on both sides
  bool aligned = reinterpret_cast<uintptr_t>(src.data_ptr()) % 16 == 0;
  for (int64_t p : dst) aligned = aligned && p % 16 == 0;
  for (int64_t i = 0; i < n; ++i) {
    const int64_t* r = g + 6 * i;
    WB_CHECK(r[0] >= 0 && r[1] >= 0 && r[2] >= 1 && r[3] >= 1 && r[4] >= r[3] && r[5] >= r[3],
             "policy_push: segment " + std::to_string(i) + " has a bad shape");
    WB_CHECK(r[0] + (r[2] - 1) * r[4] + r[3] <= src.numel(), "policy_push: segment " + std::to_string(i) + " reads past src");
    WB_CHECK(r[1] + (r[2] - 1) * r[5] + r[3] <= dst_numel, "policy_push: segment " + std::to_string(i) + " writes past dst");
    for (int k = 0; k < 6; ++k)
      if (k != 2 && r[k] % want) aligned = false;
  }
  const int vec = aligned ? want : 1;
  auto prefix = at::empty({n}, at::TensorOptions().dtype(at::kLong));
  int64_t* pf = prefix.data_ptr<int64_t>();
  int64_t total = 0;
  for (int64_t i = 0; i < n; ++i) {
    pf[i] = total;
    total += g[6 * i + 2] * (g[6 * i + 3] / vec);
  }
  auto dev = src.device();
  auto seg_d = seg.to(dev);
  auto pre_d = prefix.to(dev);
  wb::policy_push(src.data_ptr(), src_bf16 ? 1 : 0, peers_of(dst, nd), nd, dst_bf16 ? 1 : 0, seg_d.data_ptr<int64_t>(),
                  pre_d.data_ptr<int64_t>(), (int)n, total, vec, cur_stream());
  return vec;
}

void policy_signal(const std::vector<int64_t>& pads, int64_t word, int64_t value) {
  WB_CHECK(word >= 0 && word < wb::kPadWords, "policy_signal: word out of the pad");
  wb::policy_signal(peers_of(pads, (int)pads.size()), (int)pads.size(), (int)word, static_cast<uint32_t>(value),
                    cur_stream());
}

// Fused GEMM -> all-reduce / reduce-scatter, GEMM half: the tcgen05 GEMM of
// a (K-major [M, K]) and b (B(n, k) K-major [N, K] or MN-major [K, N]), with
// an optional second operand pair (LoRA), writes its bf16 partial product
// into every peer's receive buffer at element `off` (kEpiPeerBF16).
void gemm_peer(const at::Tensor& a, const at::Tensor& b, bool b_mn, int64_t N, double alpha,
               const c10::optional<at::Tensor>& a2, const c10::optional<at::Tensor>& b2,
               const std::vector<int64_t>& peers, int64_t rank, int64_t off, int64_t ldc, int64_t rs_rows) {
  check_bf16(a, "a");
  check_bf16(b, "b");
  WB_CHECK(!peers.empty() && peers.size() <= 8, "gemm_peer: 1..8 peer buffers");
  const c10::cuda::CUDAGuard guard(a.device());
  wb::GemmArgs g;
  g.A = a.data_ptr();
  g.lda = ld_of(a, "a");
  g.B = b.data_ptr();
  g.ldb = ld_of(b, "b");
  g.b_mn = b_mn;
  g.M = a.size(0);
  g.K = a.size(1);
  g.N = N;
  if (a2) {
    WB_CHECK(b2.has_value(), "gemm_peer: a2 needs b2");
    check_bf16(*a2, "a2");
    check_bf16(*b2, "b2");
    g.A2 = a2->data_ptr();
    g.lda2 = ld_of(*a2, "a2");
    g.B2 = b2->data_ptr();
    g.ldb2 = ld_of(*b2, "b2");
    g.K2 = a2->size(1);
  }
  g.epi = wb::kEpiPeerBF16;
  g.alpha = static_cast<float>(alpha);
  g.peer_world = static_cast<int>(peers.size());
  for (size_t r = 0; r < peers.size(); ++r) g.peer[r] = reinterpret_cast<void*>(peers[r]);
  g.peer_rank = static_cast<int>(rank);
  g.peer_off = off;
  g.ldc = ldc;
  g.C = g.peer[rank];
  g.peer_rs_rows = rs_rows;
  wb::gemm_bf16(g, cur_stream());
}

void slots_sum(const at::Tensor& slots, int64_t world, int64_t stride, int64_t n,
               const c10::optional<at::Tensor>& res, at::Tensor& out) {
  check_bf16(slots, "slots");
  check_bf16(out, "out");
  WB_CHECK(slots.is_contiguous() && out.is_contiguous() && slots.numel() >= (world - 1) * stride + n &&
               out.numel() >= n, "slots_sum: sizes");
  if (res) {
    check_bf16(*res, "res");
    WB_CHECK(res->is_contiguous() && res->numel() >= n, "slots_sum: res");
  }
  wb::slots_sum(slots.data_ptr(), (int)world, stride, n, res ? res->data_ptr() : nullptr, out.data_ptr(),
                cur_stream());
}

void rows_scatter(const at::Tensor& x, const at::Tensor& src_row, const at::Tensor& dst_rank, const at::Tensor& dst_row,
                  const c10::optional<at::Tensor>& scale, const std::vector<int64_t>& dst, int64_t world, int64_t ldd,
                  int64_t limit_rows) {
  check_bf16(x, "x");
  WB_CHECK(src_row.scalar_type() == at::kLong && dst_row.scalar_type() == at::kLong && dst_rank.scalar_type() == at::kInt,
           "rows_scatter: index dtypes");
  if (scale) check_f32(*scale, "scale");
  wb::rows_scatter(x.data_ptr(), ld_of(x, "x"), src_row.data_ptr<int64_t>(), dst_rank.data_ptr<int>(),
                   dst_row.data_ptr<int64_t>(), scale ? scale->data_ptr<float>() : nullptr, peers_of(dst, (int)world),
                   ldd, (int)src_row.numel(), (int)x.size(1), limit_rows, cur_stream());
}

void rows_gather_sum(const std::vector<int64_t>& src, int64_t world, int64_t lds, const at::Tensor& src_rank,
                     const at::Tensor& src_row, const c10::optional<at::Tensor>& w, int64_t k,
                     const c10::optional<at::Tensor>& res, at::Tensor& out, int64_t limit_rows) {
  WB_CHECK(src_row.scalar_type() == at::kLong && src_rank.scalar_type() == at::kInt, "rows_gather_sum: index dtypes");
  if (w) check_f32(*w, "w");
  const bool f32 = out.scalar_type() == at::kFloat;
  WB_CHECK(f32 || out.scalar_type() == at::kBFloat16, "rows_gather_sum: out bf16 or fp32");
  if (res) check_bf16(*res, "res");
  wb::rows_gather_sum(peers_of(src, (int)world), lds, src_rank.data_ptr<int>(), src_row.data_ptr<int64_t>(),
                      w ? w->data_ptr<float>() : nullptr, (int)k, res ? res->data_ptr() : nullptr,
                      res ? ld_of(*res, "res") : 0, out.data_ptr(), ld_of(out, "out"), f32, (int)out.size(0),
                      (int)out.size(1), limit_rows, cur_stream());
}

void allgather_bf16(const std::vector<int64_t>& dst, int64_t world, int64_t lo, const at::Tensor& src) {
  check_bf16(src, "src");
  wb::allgather_bf16(peers_of(dst, (int)world), (int)world, lo, src.data_ptr(), src.numel(), cur_stream());
}

void splitk_reduce(const at::Tensor& ws, int64_t S, at::Tensor& out, const c10::optional<at::Tensor>& bias,
                   const c10::optional<at::Tensor>& res, double alpha) {
  check_f32(ws, "ws");
  check_bf16(out, "out");
  const int64_t M = out.size(0), N = out.size(1);
  WB_CHECK(ws.is_contiguous() && ws.numel() == S * M * N, "splitk_reduce: workspace must be [S*M, N]");
  const c10::cuda::CUDAGuard guard(out.device());
  wb::splitk_reduce(ws.data_ptr<float>(), (int)S, M, (int)N, out.data_ptr(), ld_of(out, "out"),
                    bias ? bias->data_ptr() : nullptr, res ? res->data_ptr() : nullptr, res ? ld_of(*res, "res") : 0,
                    (float)alpha, cur_stream());
}

void nf4_dequant(const at::Tensor& codes, const at::Tensor& absmax, at::Tensor& out, const std::vector<double>& lut) {
  WB_CHECK(codes.scalar_type() == at::kByte && codes.is_cuda() && codes.is_contiguous(), "nf4_dequant: codes");
  check_f32(absmax, "absmax");
  check_bf16(out, "out");
  WB_CHECK(out.is_contiguous() && out.numel() == codes.numel() * 2 && absmax.numel() * 64 == out.numel(),
           "nf4_dequant: sizes");
  WB_CHECK(lut.size() == 16, "nf4_dequant: lut must have 16 entries");
  float l[16];
  for (int i = 0; i < 16; ++i) l[i] = static_cast<float>(lut[i]);
  wb::nf4_dequant(codes.data_ptr(), absmax.data_ptr<float>(), out.data_ptr(), out.numel(), l, cur_stream());
}

void rmsnorm_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& res,
                 const c10::optional<at::Tensor>& h_out, const at::Tensor& w, at::Tensor& y,
                 const c10::optional<at::Tensor>& rstd, double eps) {
  check_bf16(x, "x");
  check_bf16(w, "w");
  check_bf16(y, "y");
  WB_CHECK(x.is_contiguous() && y.is_contiguous(), "rmsnorm: x, y must be contiguous");
  const int H = w.numel();
  const int rows = x.numel() / H;
  const c10::cuda::CUDAGuard guard(x.device());
  wb::rmsnorm_fwd(x.data_ptr(), res ? res->data_ptr() : nullptr,
                  h_out ? h_out->data_ptr() : nullptr, w.data_ptr(), y.data_ptr(),
                  rstd ? rstd->data_ptr<float>() : nullptr, rows, H, (float)eps, cur_stream());
}

void rmsnorm_bwd(const at::Tensor& x, const at::Tensor& w, const at::Tensor& rstd,
                 const at::Tensor& dy, const c10::optional<at::Tensor>& dres, at::Tensor& dx,
                 const c10::optional<at::Tensor>& dw) {
  check_bf16(x, "x");
  check_bf16(dy, "dy");
  check_bf16(dx, "dx");
  check_f32(rstd, "rstd");
  WB_CHECK(x.is_contiguous() && dy.is_contiguous() && dx.is_contiguous(),
           "rmsnorm_bwd: tensors must be contiguous");
  const int H = w.numel();
  const int rows = x.numel() / H;
  if (dw) check_f32(*dw, "dw");
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor part;
  if (dw) part = at::empty({wb::rmsnorm_dw_splits(rows), H}, x.options().dtype(at::kFloat));
  wb::rmsnorm_bwd(x.data_ptr(), w.data_ptr(), rstd.data_ptr<float>(), dy.data_ptr(),
                  dres ? dres->data_ptr() : nullptr, dx.data_ptr(),
                  dw ? dw->data_ptr<float>() : nullptr, dw ? part.data_ptr<float>() : nullptr, rows, H,
                  cur_stream());
}

void qk_norm_rope_fwd(at::Tensor& qkv, int64_t n_q, int64_t n_k, const at::Tensor& pos,
                      const at::Tensor& inv_freq, const c10::optional<at::Tensor>& q_w,
                      const c10::optional<at::Tensor>& k_w, const c10::optional<at::Tensor>& rstd,
                      double eps) {
  check_bf16(qkv, "qkv");
  WB_CHECK(qkv.dim() == 2 && qkv.stride(1) == 1, "qk_norm_rope: qkv must be [T, W] row-major");
  WB_CHECK(pos.scalar_type() == at::kInt, "qk_norm_rope: pos must be int32");
  check_f32(inv_freq, "inv_freq");
  const c10::cuda::CUDAGuard guard(qkv.device());
  wb::qk_norm_rope_fwd(qkv.data_ptr(), qkv.stride(0), n_q, n_k, pos.data_ptr<int>(),
                       inv_freq.data_ptr<float>(), q_w ? q_w->data_ptr() : nullptr,
                       k_w ? k_w->data_ptr() : nullptr, rstd ? rstd->data_ptr<float>() : nullptr,
                       qkv.size(0), (float)eps, cur_stream());
}

void qk_norm_rope_bwd(at::Tensor& dqkv, const at::Tensor& qkv_pre, int64_t n_q, int64_t n_k,
                      const at::Tensor& pos, const at::Tensor& inv_freq,
                      const c10::optional<at::Tensor>& q_w, const c10::optional<at::Tensor>& k_w,
                      const c10::optional<at::Tensor>& rstd,
                      const c10::optional<at::Tensor>& dq_w,
                      const c10::optional<at::Tensor>& dk_w) {
  check_bf16(dqkv, "dqkv");
  const c10::cuda::CUDAGuard guard(dqkv.device());
  wb::qk_norm_rope_bwd(dqkv.data_ptr(), dqkv.stride(0), qkv_pre.data_ptr(), qkv_pre.stride(0), n_q,
                       n_k, pos.data_ptr<int>(), inv_freq.data_ptr<float>(),
                       q_w ? q_w->data_ptr() : nullptr, k_w ? k_w->data_ptr() : nullptr,
                       rstd ? rstd->data_ptr<float>() : nullptr,
                       dq_w ? dq_w->data_ptr<float>() : nullptr,
                       dk_w ? dk_w->data_ptr<float>() : nullptr, dqkv.size(0), cur_stream());
}

void swiglu_fwd(const at::Tensor& gu, at::Tensor& h) {
  check_bf16(gu, "gu");
  check_bf16(h, "h");
  WB_CHECK(gu.is_contiguous() && h.is_contiguous(), "swiglu: tensors must be contiguous");
  const int64_t I = h.size(-1);
  const c10::cuda::CUDAGuard guard(gu.device());
  wb::swiglu_fwd(gu.data_ptr(), h.data_ptr(), h.numel() / I, I, cur_stream());
}

void swiglu_bwd(const at::Tensor& gu, const at::Tensor& dh, at::Tensor& dgu) {
  check_bf16(gu, "gu");
  check_bf16(dh, "dh");
  check_bf16(dgu, "dgu");
  WB_CHECK(gu.is_contiguous() && dh.is_contiguous() && dgu.is_contiguous(),
           "swiglu_bwd: tensors must be contiguous");
  const int64_t I = dh.size(-1);
  const c10::cuda::CUDAGuard guard(gu.device());
  wb::swiglu_bwd(gu.data_ptr(), dh.data_ptr(), dgu.data_ptr(), dh.numel() / I, I, cur_stream());
}

void embedding_fwd(const at::Tensor& table, const at::Tensor& ids, at::Tensor& out) {
  check_bf16(table, "table");
  WB_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous(), "embedding: ids must be int64");
  const c10::cuda::CUDAGuard guard(table.device());
  wb::embedding_fwd(table.data_ptr(), ids.data_ptr<int64_t>(), out.data_ptr(), ids.numel(),
                    table.size(1), table.size(0), cur_stream());
}

void embedding_bwd(const at::Tensor& dy, const at::Tensor& ids, at::Tensor& dtable) {
  check_bf16(dy, "dy");
  check_f32(dtable, "dtable");
  const c10::cuda::CUDAGuard guard(dy.device());
  wb::embedding_bwd(dy.data_ptr(), ids.data_ptr<int64_t>(), dtable.data_ptr<float>(), ids.numel(),
                    dtable.size(1), dtable.size(0), cur_stream());
}

void adamw_step(at::Tensor& p, const at::Tensor& g, at::Tensor& m, at::Tensor& v,
                const c10::optional<at::Tensor>& p16, double lr, double b1, double b2, double eps,
                double wd, int64_t step, const c10::optional<at::Tensor>& gscale_dev,
                double gscale_host) {
  check_f32(p, "p");
  check_f32(g, "g");
  check_f32(m, "m");
  check_f32(v, "v");
  WB_CHECK(p.is_contiguous() && g.is_contiguous() && m.is_contiguous() && v.is_contiguous(),
           "adamw: buffers must be contiguous");
  WB_CHECK(g.numel() == p.numel() && m.numel() == p.numel() && v.numel() == p.numel(),
           "adamw: size mismatch");
  if (p16) {
    check_bf16(*p16, "p16");
    WB_CHECK(p16->numel() == p.numel() && p16->is_contiguous(), "adamw: bad p16");
  }
  const double bc1 = 1.0 - std::pow(b1, (double)step);
  const double bc2 = 1.0 - std::pow(b2, (double)step);
  const c10::cuda::CUDAGuard guard(p.device());
  wb::adamw_step(p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(),
                 v.data_ptr<float>(), p16 ? p16->data_ptr() : nullptr, p.numel(), (float)lr,
                 (float)b1, (float)b2, (float)eps, (float)wd, (float)bc1, (float)bc2,
                 gscale_dev ? gscale_dev->data_ptr<float>() : nullptr, (float)gscale_host,
                 cur_stream());
}

void adamw8_step(at::Tensor& p, const at::Tensor& g, at::Tensor& m8, at::Tensor& v8, at::Tensor& am,
                 at::Tensor& av, const c10::optional<at::Tensor>& p16, double lr, double b1, double b2, double eps,
                 double wd, int64_t step, const c10::optional<at::Tensor>& gscale_dev, double gscale_host) {
  check_f32(p, "p");
  check_f32(g, "g");
  check_f32(am, "am");
  check_f32(av, "av");
  const int64_t n = p.numel();
  WB_CHECK(p.is_contiguous() && g.is_contiguous() && m8.is_contiguous() && v8.is_contiguous(),
           "adamw8: buffers must be contiguous");
  WB_CHECK(m8.scalar_type() == at::kChar && v8.scalar_type() == at::kByte, "adamw8: m8 int8, v8 uint8");
  WB_CHECK(g.numel() == n && m8.numel() == n && v8.numel() == n, "adamw8: size mismatch");
  WB_CHECK(am.numel() >= (n + 255) / 256 && av.numel() >= (n + 255) / 256, "adamw8: scale buffers too small");
  if (p16) {
    check_bf16(*p16, "p16");
    WB_CHECK(p16->numel() == n && p16->is_contiguous(), "adamw8: bad p16");
  }
  const double bc1 = 1.0 - std::pow(b1, (double)step);
  const double bc2 = 1.0 - std::pow(b2, (double)step);
  const c10::cuda::CUDAGuard guard(p.device());
  wb::adamw8_step(p.data_ptr<float>(), g.data_ptr<float>(), m8.data_ptr<int8_t>(), v8.data_ptr<uint8_t>(),
                  am.data_ptr<float>(), av.data_ptr<float>(), p16 ? p16->data_ptr() : nullptr, n, (float)lr,
                  (float)b1, (float)b2, (float)eps, (float)wd, (float)bc1, (float)bc2,
                  gscale_dev ? gscale_dev->data_ptr<float>() : nullptr, (float)gscale_host, cur_stream());
}

// Managed ("paged") device memory: pages migrate to host memory under device
// memory pressure and back on access; preferred location is `device`.
at::Tensor managed_empty(int64_t nbytes, int64_t device) {
  void* ptr = nullptr;
  WB_CHECK(cudaMallocManaged(&ptr, (size_t)std::max<int64_t>(nbytes, 1)) == cudaSuccess, "cudaMallocManaged failed");
  cudaMemLocation loc{};
  loc.type = cudaMemLocationTypeDevice;
  loc.id = (int)device;
  cudaMemAdvise(ptr, (size_t)std::max<int64_t>(nbytes, 1), cudaMemAdviseSetPreferredLocation, loc);
  cudaMemset(ptr, 0, (size_t)std::max<int64_t>(nbytes, 1));
  auto opts = at::TensorOptions().dtype(at::kByte).device(at::kCUDA, static_cast<c10::DeviceIndex>(device));
  return at::from_blob(ptr, {nbytes}, [](void* q) { cudaFree(q); }, opts);
}

void sumsq(const at::Tensor& x, at::Tensor& out) {
  check_f32(x, "x");
  check_f32(out, "out");
  WB_CHECK(x.is_contiguous(), "sumsq: x must be contiguous");
  const c10::cuda::CUDAGuard guard(x.device());
  wb::sumsq(x.data_ptr<float>(), x.numel(), out.data_ptr<float>(), cur_stream());
}

void clip_factor(const at::Tensor& sumsq_v, double max_norm, at::Tensor& out) {
  const c10::cuda::CUDAGuard guard(sumsq_v.device());
  wb::clip_factor(sumsq_v.data_ptr<float>(), (float)max_norm, out.data_ptr<float>(), cur_stream());
}

void softmax_stats(const at::Tensor& z, const c10::optional<at::Tensor>& target, double inv_tau,
                   at::Tensor& lse, const c10::optional<at::Tensor>& lp,
                   const c10::optional<at::Tensor>& ent) {
  check_bf16(z, "z");
  WB_CHECK(z.dim() == 2 && z.stride(1) == 1, "softmax_stats: z must be [rows, V] row-major");
  check_f32(lse, "lse");
  const c10::cuda::CUDAGuard guard(z.device());
  wb::softmax_stats(z.data_ptr(), z.stride(0), z.size(0), z.size(1),
                    target ? target->data_ptr<int64_t>() : nullptr, (float)inv_tau,
                    lse.data_ptr<float>(), lp ? lp->data_ptr<float>() : nullptr,
                    ent ? ent->data_ptr<float>() : nullptr, cur_stream());
}

void softmax_grad(at::Tensor& z, const c10::optional<at::Tensor>& target, double inv_tau,
                  const at::Tensor& lse, const c10::optional<at::Tensor>& ent,
                  const c10::optional<at::Tensor>& dlp, const c10::optional<at::Tensor>& dent) {
  check_bf16(z, "z");
  WB_CHECK(z.dim() == 2 && z.stride(1) == 1, "softmax_grad: z must be [rows, V] row-major");
  const c10::cuda::CUDAGuard guard(z.device());
  wb::softmax_grad(z.data_ptr(), z.stride(0), z.size(0), z.size(1),
                   target ? target->data_ptr<int64_t>() : nullptr, (float)inv_tau,
                   lse.data_ptr<float>(), ent ? ent->data_ptr<float>() : nullptr,
                   dlp ? dlp->data_ptr<float>() : nullptr, dent ? dent->data_ptr<float>() : nullptr,
                   cur_stream());
}

// q/k/v: [T, H, 128] views whose head and dim strides are (128, 1).
static int64_t head_row_stride(const at::Tensor& t, const char* name) {
  check_bf16(t, name);
  WB_CHECK(t.dim() == 3 && t.size(2) == 128, std::string(name) + " must be [T, H, 128]");
  WB_CHECK(t.stride(2) == 1 && t.stride(1) == 128, std::string(name) + " must have head stride 128, dim stride 1");
  return t.stride(0);
}

static wb::AttnArgs attn_args(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                              const at::Tensor& cu, int64_t max_seqlen, bool causal, double scale,
                              const c10::optional<at::Tensor>& cu_k = c10::nullopt, int64_t max_seqlen_k = 0) {
  WB_CHECK(causal, "attention: only causal attention is implemented");
  WB_CHECK(cu.scalar_type() == at::kInt && cu.is_cuda() && cu.is_contiguous(), "attention: cu_seqlens must be int32 CUDA");
  wb::AttnArgs a;
  a.q = q.data_ptr();
  a.k = k.data_ptr();
  a.v = v.data_ptr();
  a.q_row = head_row_stride(q, "q");
  a.k_row = head_row_stride(k, "k");
  a.v_row = head_row_stride(v, "v");
  a.T = q.size(0);
  a.Hq = q.size(1);
  a.Hk = k.size(1);
  a.cu_seqlens = cu.data_ptr<int>();
  a.nseq = cu.numel() - 1;
  a.max_seqlen = max_seqlen;
  a.scale = static_cast<float>(scale);
  if (cu_k) {
    WB_CHECK(cu_k->scalar_type() == at::kInt && cu_k->is_cuda() && cu_k->is_contiguous() && cu_k->numel() == cu.numel(),
             "attention: cu_seqlens_k must be int32 CUDA with one entry per cu_seqlens entry");
    WB_CHECK(v.size(0) == k.size(0) && v.size(1) == a.Hk, "attention: k/v shape mismatch");
    a.cu_seqlens_k = cu_k->data_ptr<int>();
    a.max_seqlen_k = max_seqlen_k;
    a.Tk = k.size(0);
  } else {
    WB_CHECK(k.size(0) == a.T && v.size(0) == a.T && v.size(1) == a.Hk, "attention: k/v shape mismatch");
  }
  return a;
}

void attn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& cu,
              int64_t max_seqlen, bool causal, double scale, at::Tensor& out, at::Tensor& lse,
              const c10::optional<at::Tensor>& cu_k, int64_t max_seqlen_k) {
  const c10::cuda::CUDAGuard guard(q.device());
  wb::AttnArgs a = attn_args(q, k, v, cu, max_seqlen, causal, scale, cu_k, max_seqlen_k);
  check_bf16(out, "out");
  WB_CHECK(out.is_contiguous() && out.sizes() == q.sizes(), "attention: out must be contiguous [T, Hq, 128]");
  check_f32(lse, "lse");
  WB_CHECK(lse.is_contiguous() && lse.size(0) == a.Hq && lse.size(1) == a.T, "attention: lse must be [Hq, T]");
  a.o = out.data_ptr();
  a.o_row = out.stride(0);
  a.lse = lse.data_ptr<float>();
  if (a.T == 0 || a.nseq == 0) return;
  wb::attn_fwd(a, cur_stream());
}

void attn_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
              const at::Tensor& out, const at::Tensor& lse, const at::Tensor& cu, int64_t max_seqlen, bool causal,
              double scale, at::Tensor& dq, at::Tensor& dk, at::Tensor& dv, const c10::optional<at::Tensor>& cu_k,
              int64_t max_seqlen_k) {
  const c10::cuda::CUDAGuard guard(q.device());
  wb::AttnBwdArgs b;
  b.f = attn_args(q, k, v, cu, max_seqlen, causal, scale, cu_k, max_seqlen_k);
  check_bf16(dout, "dout");
  WB_CHECK(dout.is_contiguous() && dout.sizes() == q.sizes(), "attention: dout must be contiguous [T, Hq, 128]");
  WB_CHECK(out.sizes() == q.sizes() && out.stride(2) == 1 && out.stride(1) == 128, "attention: bad out");
  b.f.o = const_cast<void*>(out.data_ptr());
  b.f.o_row = out.stride(0);
  b.f.lse = const_cast<float*>(lse.data_ptr<float>());
  for (auto* t : {&dq, &dk, &dv}) WB_CHECK(t->is_contiguous() && t->scalar_type() == at::kBFloat16, "attention: grads must be contiguous bf16");
  b.dout = dout.data_ptr();
  b.dq = dq.data_ptr();
  b.dk = dk.data_ptr();
  b.dv = dv.data_ptr();
  at::Tensor delta = at::empty({b.f.Hq, b.f.T}, q.options().dtype(at::kFloat));
  b.delta = delta.data_ptr<float>();
  at::Tensor pdk, pdv;
  WB_CHECK(dk.sizes() == k.sizes() && dv.sizes() == v.sizes(), "attention: dk/dv must match k/v");
  if (b.f.Hq != b.f.Hk) {
    const int64_t Tk = k.size(0);
    pdk = at::empty({Tk, b.f.Hq, 128}, q.options().dtype(at::kFloat));
    pdv = at::empty({Tk, b.f.Hq, 128}, q.options().dtype(at::kFloat));
    b.part_dk = pdk.data_ptr<float>();
    b.part_dv = pdv.data_ptr<float>();
  }
  if (b.f.T == 0 || b.f.nseq == 0) return;
  wb::attn_bwd(b, cur_stream());
}

void kv_append(const at::Tensor& k, const at::Tensor& v, at::Tensor& k_cache, at::Tensor& v_cache,
               const at::Tensor& slot) {
  // k, v: [T, Hk, 128] views; caches [num_blocks, Hk, block_size, 128]; slot int32 [T]
  check_bf16(k, "k");
  check_bf16(v, "v");
  WB_CHECK(k.stride(2) == 1 && k.stride(1) == 128 && v.stride(2) == 1 && v.stride(1) == 128, "kv_append: bad k/v layout");
  WB_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous(), "kv_append: caches must be contiguous");
  WB_CHECK(slot.scalar_type() == at::kInt && slot.is_contiguous(), "kv_append: slot must be int32");
  const c10::cuda::CUDAGuard guard(k.device());
  wb::kv_append(k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0), k_cache.data_ptr(), v_cache.data_ptr(),
                slot.data_ptr<int>(), k.size(0), k.size(1), k_cache.size(2), cur_stream());
}

void decode_attention(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                      const at::Tensor& block_tables, const at::Tensor& ctx_lens, at::Tensor& out, int64_t splits,
                      double scale) {
  check_bf16(q, "q");
  WB_CHECK(q.dim() == 3 && q.stride(2) == 1 && q.stride(1) == 128 && q.size(2) == 128, "decode_attention: q must be [B, Hq, 128]");
  WB_CHECK(out.dim() == 3 && out.stride(2) == 1 && out.stride(1) == 128, "decode_attention: bad out");
  WB_CHECK(block_tables.scalar_type() == at::kInt && block_tables.is_contiguous(), "decode_attention: block_tables int32");
  WB_CHECK(ctx_lens.scalar_type() == at::kInt, "decode_attention: ctx_lens int32");
  const c10::cuda::CUDAGuard guard(q.device());
  wb::DecodeArgs a;
  a.q = q.data_ptr();
  a.q_row = q.stride(0);
  a.k_cache = k_cache.data_ptr();
  a.v_cache = v_cache.data_ptr();
  a.block_tables = block_tables.data_ptr<int>();
  a.max_blocks = block_tables.size(1);
  a.ctx_lens = ctx_lens.data_ptr<int>();
  a.out = out.data_ptr();
  a.out_row = out.stride(0);
  a.nseq = q.size(0);
  a.Hq = q.size(1);
  a.Hk = k_cache.size(1);  // [num_blocks, Hk, block_size, 128]
  a.block_size = k_cache.size(2);
  a.cache_rows = k_cache.size(0) * k_cache.size(2);
  a.splits = std::max<int64_t>(1, splits);
  a.scale = (float)scale;
  at::Tensor po, pml;
  if (a.splits > 1) {
    po = at::empty({a.nseq, a.Hq, a.splits, 128}, q.options().dtype(at::kFloat));
    pml = at::empty({a.nseq, a.Hq, a.splits, 2}, q.options().dtype(at::kFloat));
    a.part_o = po.data_ptr<float>();
    a.part_ml = pml.data_ptr<float>();
  }
  wb::decode_attention(a, cur_stream());
}

void sample_tokens(const at::Tensor& z, const at::Tensor& inv_tau, const c10::optional<at::Tensor>& thresh,
                   double min_p, int64_t seed, const c10::optional<at::Tensor>& row_ids, at::Tensor& out_tok,
                   at::Tensor& out_lp, const c10::optional<at::Tensor>& seed_dev) {
  check_bf16(z, "z");
  WB_CHECK(z.dim() == 2 && z.stride(1) == 1, "sample_tokens: z must be [B, V] row-major");
  check_f32(inv_tau, "inv_tau");
  const c10::cuda::CUDAGuard guard(z.device());
  wb::sample_tokens(z.data_ptr(), z.stride(0), z.size(0), z.size(1), inv_tau.data_ptr<float>(),
                    thresh ? thresh->data_ptr<float>() : nullptr, (float)min_p, (uint64_t)seed,
                    row_ids ? row_ids->data_ptr<int64_t>() : nullptr, out_tok.data_ptr<int64_t>(),
                    out_lp.data_ptr<float>(), cur_stream(), seed_dev ? seed_dev->data_ptr<int64_t>() : nullptr);
}

void sample_thresholds(const at::Tensor& z, const c10::optional<at::Tensor>& top_k,
                       const c10::optional<at::Tensor>& top_p, const c10::optional<at::Tensor>& inv_tau,
                       at::Tensor& out) {
  check_bf16(z, "z");
  WB_CHECK(z.dim() == 2 && z.stride(1) == 1, "sample_thresholds: z must be [B, V] row-major");
  check_f32(out, "out");
  WB_CHECK(out.numel() >= z.size(0), "sample_thresholds: out too small");
  if (top_k) WB_CHECK(top_k->scalar_type() == at::kInt && top_k->is_contiguous(), "sample_thresholds: top_k int32");
  if (top_p) check_f32(*top_p, "top_p");
  if (inv_tau) check_f32(*inv_tau, "inv_tau");
  const c10::cuda::CUDAGuard guard(z.device());
  wb::sample_thresholds(z.data_ptr(), z.stride(0), (int)z.size(0), (int)z.size(1),
                        top_k ? top_k->data_ptr<int32_t>() : nullptr, top_p ? top_p->data_ptr<float>() : nullptr,
                        inv_tau ? inv_tau->data_ptr<float>() : nullptr, out.data_ptr<float>(), cur_stream());
}

void decode_advance(const at::Tensor& tok, const at::Tensor& lp, at::Tensor& ids, at::Tensor& pos, at::Tensor& ctx,
                    at::Tensor& slots, const at::Tensor& bt, int64_t block_size, at::Tensor& win_tok,
                    at::Tensor& win_lp, at::Tensor& step, at::Tensor& seed) {
  WB_CHECK(tok.scalar_type() == at::kLong && ids.scalar_type() == at::kLong && seed.scalar_type() == at::kLong,
           "decode_advance: tok/ids/seed int64");
  WB_CHECK(pos.scalar_type() == at::kInt && ctx.scalar_type() == at::kInt && slots.scalar_type() == at::kInt &&
               bt.scalar_type() == at::kInt && step.scalar_type() == at::kInt, "decode_advance: int32 state");
  WB_CHECK(bt.dim() == 2 && bt.size(0) >= tok.size(0) && win_tok.size(0) >= tok.size(0), "decode_advance: shapes");
  const c10::cuda::CUDAGuard guard(tok.device());
  wb::decode_advance(tok.data_ptr<int64_t>(), lp.data_ptr<float>(), ids.data_ptr<int64_t>(), pos.data_ptr<int32_t>(),
                     ctx.data_ptr<int32_t>(), slots.data_ptr<int32_t>(), bt.data_ptr<int32_t>(), (int)bt.size(1),
                     (int)block_size, win_tok.data_ptr<int64_t>(), win_lp.data_ptr<float>(), (int)win_tok.size(1),
                     step.data_ptr<int32_t>(), seed.data_ptr<int64_t>(), (int)tok.size(0), cur_stream());
}

static void check_i32(const at::Tensor& t, const char* name) {
  WB_CHECK(t.is_cuda() && t.scalar_type() == at::kInt && t.is_contiguous(), std::string(name) + " must be int32 CUDA");
}
static void check_i64(const at::Tensor& t, const char* name) {
  WB_CHECK(t.is_cuda() && t.scalar_type() == at::kLong && t.is_contiguous(), std::string(name) + " must be int64 CUDA");
}

void moe_route(const at::Tensor& logits, int64_t k, bool norm_topk, bool bf16_logits, at::Tensor& probs,
               at::Tensor& topi, at::Tensor& topv, at::Tensor& w, at::Tensor& ssum, at::Tensor& counts) {
  check_f32(logits, "logits");
  WB_CHECK(logits.dim() == 2 && logits.is_contiguous(), "moe_route: logits [T, E] contiguous");
  const int64_t T = logits.size(0), E = logits.size(1);
  check_f32(probs, "probs");
  check_f32(topv, "topv");
  check_f32(w, "w");
  check_f32(ssum, "ssum");
  check_i64(topi, "topi");
  check_i32(counts, "counts");
  WB_CHECK(probs.numel() == T * E && topi.numel() == T * k && topv.numel() == T * k && w.numel() == T * k &&
               ssum.numel() == T && counts.numel() >= E, "moe_route: output sizes");
  const c10::cuda::CUDAGuard guard(logits.device());
  wb::moe_route(logits.data_ptr<float>(), (int)T, (int)E, (int)k, norm_topk, bf16_logits, probs.data_ptr<float>(),
                topi.data_ptr<int64_t>(), topv.data_ptr<float>(), w.data_ptr<float>(), ssum.data_ptr<float>(),
                counts.data_ptr<int32_t>(), cur_stream());
}

void moe_layout(const at::Tensor& allc, int64_t ep, int64_t me, int64_t pad, int64_t cap_rows, at::Tensor& base,
                at::Tensor& tile_group, at::Tensor& k_start, at::Tensor& k_len, at::Tensor& n_recv, at::Tensor& rows,
                at::Tensor& overflow) {
  check_i32(allc, "allc");
  check_i64(base, "base");
  check_i32(tile_group, "tile_group");
  check_i32(k_start, "k_start");
  check_i32(k_len, "k_len");
  check_i32(n_recv, "n_recv");
  check_i32(rows, "rows");
  check_i32(overflow, "overflow");
  const int64_t E = base.numel();
  WB_CHECK(allc.numel() >= ep * E && ep > 0 && E % ep == 0 && me >= 0 && me < ep, "moe_layout: bad counts table");
  WB_CHECK(k_start.numel() >= E / ep && k_len.numel() >= E / ep && n_recv.numel() >= E / ep, "moe_layout: sizes");
  int dev = 0;
  cudaGetDevice(&dev);
  const c10::cuda::CUDAGuard guard(allc.device());
  wb::moe_layout(allc.data_ptr<int32_t>(), (int)ep, (int)me, (int)E, (int)pad, cap_rows, (int)tile_group.numel(),
                 base.data_ptr<int64_t>(), tile_group.data_ptr<int32_t>(), k_start.data_ptr<int32_t>(),
                 k_len.data_ptr<int32_t>(), n_recv.data_ptr<int32_t>(), rows.data_ptr<int32_t>(),
                 overflow.data_ptr<int32_t>(), wb::error_word(allc.get_device()), cur_stream());
}

void moe_copy_rows(const at::Tensor& topi, int64_t E, int64_t El, const at::Tensor& base, at::Tensor& dst_row,
                   at::Tensor& dst_rank) {
  check_i64(topi, "topi");
  check_i64(base, "base");
  check_i64(dst_row, "dst_row");
  check_i32(dst_rank, "dst_rank");
  WB_CHECK(dst_row.numel() == topi.numel() && dst_rank.numel() == topi.numel() && base.numel() >= E,
           "moe_copy_rows: sizes");
  const c10::cuda::CUDAGuard guard(topi.device());
  wb::moe_copy_rows(topi.data_ptr<int64_t>(), (int)topi.numel(), (int)E, (int)El, base.data_ptr<int64_t>(),
                    dst_row.data_ptr<int64_t>(), dst_rank.data_ptr<int32_t>(), cur_stream());
}

void moe_zero_pad(at::Tensor& x, const at::Tensor& k_start, const at::Tensor& k_len, const at::Tensor& n_recv,
                  const c10::optional<at::Tensor>& overflow) {
  check_bf16(x, "x");
  WB_CHECK(x.dim() == 2 && x.stride(1) == 1, "moe_zero_pad: x [R, H] row-major");
  check_i32(k_start, "k_start");
  const c10::cuda::CUDAGuard guard(x.device());
  wb::moe_zero_pad(x.data_ptr(), x.stride(0), (int)x.size(1), (int)k_start.numel(), k_start.data_ptr<int32_t>(),
                   k_len.data_ptr<int32_t>(), n_recv.data_ptr<int32_t>(),
                   overflow ? overflow->data_ptr<int32_t>() : nullptr, cur_stream());
}

void moe_put_counts(const std::vector<int64_t>& dst, int64_t world, int64_t me, const at::Tensor& cnt) {
  check_i32(cnt, "cnt");
  const c10::cuda::CUDAGuard guard(cnt.device());
  wb::moe_put_counts(peers_of(dst, (int)world), (int)world, (int)me, (int)cnt.numel(), cnt.data_ptr<int32_t>(),
                     cur_stream());
}

int64_t read_error(int64_t device) { return wb::read_error_word((int)device); }
void clear_error(int64_t device) { wb::clear_error_word((int)device); }

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "wavelet_b200 sm_100a kernels";
  m.def("gemm", &gemm, "tcgen05 bf16 GEMM", py::arg("a"), py::arg("a_mn"), py::arg("b"),
        py::arg("b_mn"), py::arg("c"), py::arg("epi") = 0, py::arg("alpha") = 1.0,
        py::arg("bias") = py::none(), py::arg("res") = py::none());
  m.def("gemm_grouped", &gemm_grouped);
  m.def("gemm_ex", &gemm_ex);
  m.def("nf4_dequant", &nf4_dequant);
  m.def("splitk_reduce", &splitk_reduce);
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("qk_norm_rope_fwd", &qk_norm_rope_fwd);
  m.def("qk_norm_rope_bwd", &qk_norm_rope_bwd);
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("embedding_fwd", &embedding_fwd);
  m.def("embedding_bwd", &embedding_bwd);
  m.def("adamw_step", &adamw_step);
  m.def("sumsq", &sumsq);
  m.def("adamw8_step", &adamw8_step);
  m.def("managed_empty", &managed_empty);
  m.def("clip_factor", &clip_factor);
  m.def("softmax_stats", &softmax_stats);
  m.def("softmax_grad", &softmax_grad);
  m.def("attn_fwd", &attn_fwd);
  m.def("attn_bwd", &attn_bwd);
  m.def("kv_append", &kv_append);
  m.def("decode_attention", &decode_attention);
  m.def("sample_tokens", &sample_tokens, py::arg("z"), py::arg("inv_tau"), py::arg("thresh"), py::arg("min_p"),
        py::arg("seed"), py::arg("row_ids"), py::arg("out_tok"), py::arg("out_lp"), py::arg("seed_dev") = py::none());
  m.def("decode_advance", &decode_advance);
  m.def("sample_thresholds", &sample_thresholds, py::arg("z"), py::arg("top_k"), py::arg("top_p"),
        py::arg("inv_tau"), py::arg("out"));
  m.def("fabric_malloc", &fabric_malloc_);
  m.def("fabric_free", &fabric_free_);
  m.def("fabric_export", &fabric_export_);
  m.def("fabric_import", &fabric_import_);
  m.def("fabric_close", &fabric_close_);
  m.def("from_ptr", &from_ptr);
  m.def("peer_barrier", &peer_barrier);
  m.def("rs_sum_sumsq", &rs_sum_sumsq, py::arg("grads"), py::arg("world"), py::arg("lo"), py::arg("n"),
        py::arg("scale"), py::arg("out"), py::arg("stats"), py::arg("w_end") = 0, py::arg("w_lo") = 1.0);
  m.def("norm_exchange", &norm_exchange);
  m.def("adamw_allgather", &adamw_allgather);
  m.def("allgather_bf16", &allgather_bf16);
  m.def("rows_scatter", &rows_scatter, py::arg("x"), py::arg("src_row"), py::arg("dst_rank"), py::arg("dst_row"),
        py::arg("scale"), py::arg("dst"), py::arg("world"), py::arg("ldd"), py::arg("limit_rows") = -1);
  m.def("gather_from_peers", &gather_from_peers);
  m.def("gemm_peer", &gemm_peer);
  m.def("slots_sum", &slots_sum);
  m.def("rows_gather_sum", &rows_gather_sum, py::arg("src"), py::arg("world"), py::arg("lds"), py::arg("src_rank"),
        py::arg("src_row"), py::arg("w"), py::arg("k"), py::arg("res"), py::arg("out"), py::arg("limit_rows") = -1);
  m.def("read_error", &read_error);
  m.def("moe_route", &moe_route);
  m.def("moe_layout", &moe_layout);
  m.def("moe_copy_rows", &moe_copy_rows);
  m.def("moe_zero_pad", &moe_zero_pad);
  m.def("moe_put_counts", &moe_put_counts);
  m.def("policy_push", &policy_push, py::arg("src"), py::arg("dst"), py::arg("dst_numel"), py::arg("dst_bf16"),
        py::arg("seg"));
  m.def("policy_signal", &policy_signal);
  m.def("launch_count", []() { return wb::launch_count(); },
        "kernels launched by this library since it was loaded (every launch site counts one)");
  m.def("note_launches", [](int64_t n) { wb::note_launches(n); },
        "count n launches made outside the launch sites (kernels replayed from a captured graph)");
  m.def("clear_error", &clear_error);
  m.attr("EPI_BF16") = (int)wb::kEpiBF16;
  m.attr("EPI_F32") = (int)wb::kEpiF32;
  m.attr("EPI_F32_ACC") = (int)wb::kEpiF32Acc;
}
