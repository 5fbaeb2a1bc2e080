// Python bindings of the sm_100a kernels (module lunaflux_b200._C).
//
// Every entry launches on the current torch CUDA stream and allocates nothing,
// so all of them can be captured inside a CUDA graph.  Shapes, dtypes and
// strides are checked here; kernels never see an operand they cannot handle.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "kernels/attention.h"
#include "kernels/elementwise.h"
#include "kernels/gemm_bf16.h"
#include "kernels/gemm_fp8.h"
#include "kernels/moe.h"
#include "kernels/moe_a2a.h"
#include "kernels/sp_gather.h"
#include "kernels/runtime.h"

namespace lf {
namespace rt {
pybind11::dict device_report();
}
}  // namespace lf

namespace {

#define LF_CHECK(cond, msg) TORCH_CHECK(cond, "lunaflux: ", msg)

void check_cuda(const at::Tensor& t, const char* name) {
  LF_CHECK(t.is_cuda(), std::string(name) + " must be a CUDA tensor");
}
void check_rowmajor(const at::Tensor& t, const char* name) {
  LF_CHECK(t.dim() == 2 && t.stride(1) == 1, std::string(name) + " must be 2-D with unit inner stride");
}

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void gemm(const at::Tensor& A, const at::Tensor& B, at::Tensor& D, int64_t epi, int64_t bn,
          c10::optional<at::Tensor> ws) {
  check_cuda(A, "A");
  check_cuda(B, "B");
  check_cuda(D, "D");
  check_rowmajor(A, "A");
  check_rowmajor(B, "B");
  check_rowmajor(D, "D");
  LF_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm operands must be bf16");
  LF_CHECK(A.size(1) == B.size(1), "gemm K mismatch");
  const int M = A.size(0), N = B.size(0), K = A.size(1);
  if (epi == 2) {
    LF_CHECK(D.size(0) == M && D.size(1) == N / 2, "SwiGLU output must be [M, N/2]");
    LF_CHECK(D.scalar_type() == at::kBFloat16, "SwiGLU output must be bf16");
  } else {
    LF_CHECK(D.size(0) == M && D.size(1) == N, "gemm output must be [M, N]");
    LF_CHECK(D.scalar_type() == (epi == 1 ? at::kFloat : at::kBFloat16), "gemm output dtype mismatch");
  }
  c10::cuda::CUDAGuard g(A.device());
  lf::gemm::GemmArgs a{A.data_ptr(), B.data_ptr(), D.data_ptr(), M, N, K, A.stride(0), B.stride(0), D.stride(0)};
  float* wsp = nullptr;
  int64_t ws_elems = 0;
  if (ws.has_value()) {
    LF_CHECK(ws->is_cuda() && ws->scalar_type() == at::kFloat && ws->is_contiguous(), "gemm workspace must be fp32");
    wsp = ws->data_ptr<float>();
    ws_elems = ws->numel();
  }
  lf::gemm::run(a, (int)epi, (int)bn, stream(), wsp, ws_elems);
}

// GEMM + all-reduce over the tensor-parallel group.  Pointers are raw device
// addresses of this rank's symmetric slot, its multicast address (0 if none)
// and every rank's slot; the same for the int32 arrival counters.
static lf::gemm::ArArgs make_ar(int64_t local, int64_t mc, const std::vector<int64_t>& peers, int64_t out_mc,
                                const std::vector<int64_t>& out_peers, int64_t cnt_local, int64_t cnt_mc,
                                const std::vector<int64_t>& cnt_peers, int64_t rank, int64_t cnt_capacity,
                                int64_t trace) {
  LF_CHECK(!peers.empty() && peers.size() <= (size_t)lf::gemm::kMaxRanks && out_peers.size() == peers.size() &&
               cnt_peers.size() == peers.size(),
           "fused all-reduce: peer lists");
  LF_CHECK(rank >= 0 && rank < (int64_t)peers.size(), "fused all-reduce: rank");
  lf::gemm::ArArgs ar{};
  ar.local = reinterpret_cast<__nv_bfloat16*>(local);
  ar.mc = reinterpret_cast<__nv_bfloat16*>(mc);
  ar.out_mc = reinterpret_cast<__nv_bfloat16*>(out_mc);
  for (size_t i = 0; i < peers.size(); ++i) {
    ar.peer[i] = reinterpret_cast<const __nv_bfloat16*>(peers[i]);
    ar.out_peer[i] = reinterpret_cast<__nv_bfloat16*>(out_peers[i]);
    ar.cnt_peer[i] = reinterpret_cast<int*>(cnt_peers[i]);
  }
  ar.cnt_local = reinterpret_cast<int*>(cnt_local);
  ar.cnt_mc = reinterpret_cast<int*>(cnt_mc);
  ar.rank = (int)rank;
  ar.world = (int)peers.size();
  ar.cnt_capacity = (int)cnt_capacity;
  ar.trace = reinterpret_cast<unsigned long long*>(trace);
  return ar;
}

// Result region (out_peers[rank], [M, N] row-major) = sum over ranks of A . B^T.
void gemm_allreduce(const at::Tensor& A, const at::Tensor& B, c10::optional<at::Tensor> ws, int64_t local, int64_t mc,
                    std::vector<int64_t> peers, int64_t out_mc, std::vector<int64_t> out_peers, int64_t cnt_local,
                    int64_t cnt_mc, std::vector<int64_t> cnt_peers, int64_t rank, int64_t cnt_capacity,
                    int64_t trace) {
  check_rowmajor(A, "A");
  check_rowmajor(B, "B");
  LF_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm_allreduce is bf16");
  const int M = A.size(0), N = B.size(0), K = A.size(1);
  lf::gemm::ArArgs ar =
      make_ar(local, mc, peers, out_mc, out_peers, cnt_local, cnt_mc, cnt_peers, rank, cnt_capacity, trace);
  float* wsp = nullptr;
  int64_t ws_elems = 0;
  if (ws.has_value()) {
    wsp = ws->data_ptr<float>();
    ws_elems = ws->numel();
  }
  c10::cuda::CUDAGuard g(A.device());
  lf::gemm::GemmArgs a{A.data_ptr(), B.data_ptr(), ar.out_peer[rank], M, N, K, A.stride(0), B.stride(0), N};
  lf::gemm::run_allreduce(a, ar, stream(), wsp, ws_elems);
}

// Rows [rank * M / world, (rank + 1) * M / world) of the sum over ranks of
// A . B^T into out_local [M / world, N] (the owner-computes tile path with the
// owner keeping its rows; M / world a multiple of 128).
void gemm_reduce_scatter(const at::Tensor& A, const at::Tensor& B, at::Tensor& out_local, int64_t local, int64_t mc,
                         std::vector<int64_t> peers, int64_t out_mc, std::vector<int64_t> out_peers,
                         int64_t cnt_local, int64_t cnt_mc, std::vector<int64_t> cnt_peers, int64_t rank,
                         int64_t cnt_capacity, int64_t trace) {
  check_rowmajor(A, "A");
  check_rowmajor(B, "B");
  LF_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16 &&
               out_local.scalar_type() == at::kBFloat16 && out_local.is_contiguous(),
           "gemm_reduce_scatter is bf16, contiguous output");
  const int M = A.size(0), N = B.size(0), K = A.size(1);
  lf::gemm::ArArgs ar =
      make_ar(local, mc, peers, out_mc, out_peers, cnt_local, cnt_mc, cnt_peers, rank, cnt_capacity, trace);
  LF_CHECK(M % ar.world == 0 && out_local.size(0) == M / ar.world && out_local.size(1) == N,
           "gemm_reduce_scatter: out_local must be [M / world, N]");
  ar.rs_rows = M / ar.world;
  ar.rs_out = reinterpret_cast<__nv_bfloat16*>(out_local.data_ptr());
  c10::cuda::CUDAGuard g(A.device());
  lf::gemm::GemmArgs a{A.data_ptr(), B.data_ptr(), ar.out_peer[rank], M, N, K, A.stride(0), B.stride(0), N};
  lf::gemm::run_reduce_scatter(a, ar, stream());
}

// ---------------------------------------------------------------------------
// Expert-parallel dispatch / combine (moe_a2a.cu).  Pointer lists: one entry
// per rank, the symmetric buffer as mapped on that rank.
static lf::a2a::Args make_a2a(const std::vector<int64_t>& recv_x, const std::vector<int64_t>& recv_meta,
                              const std::vector<int64_t>& recv_flag, const std::vector<int64_t>& comb_y,
                              const std::vector<int64_t>& comb_flag, const at::Tensor& state,
                              const at::Tensor& counts, int64_t rank, int64_t experts_local, int64_t topk,
                              int64_t cap, int64_t hidden) {
  const size_t W = recv_x.size();
  LF_CHECK(W >= 1 && W <= (size_t)lf::a2a::kMaxRanks && recv_meta.size() == W && recv_flag.size() == W &&
               comb_y.size() == W && comb_flag.size() == W,
           "moe all-to-all: peer lists");
  LF_CHECK(state.is_cuda() && state.scalar_type() == at::kInt && state.numel() >= 4, "moe all-to-all: state");
  LF_CHECK(counts.is_cuda() && counts.scalar_type() == at::kInt && counts.numel() >= (int64_t)(2 * W),
           "moe all-to-all: counts");
  lf::a2a::Args a{};
  for (size_t i = 0; i < W; ++i) {
    a.recv_x[i] = reinterpret_cast<__nv_bfloat16*>(recv_x[i]);
    a.recv_meta[i] = reinterpret_cast<int2*>(recv_meta[i]);
    a.recv_flag[i] = reinterpret_cast<unsigned long long*>(recv_flag[i]);
    a.comb_y[i] = reinterpret_cast<__nv_bfloat16*>(comb_y[i]);
    a.comb_flag[i] = reinterpret_cast<unsigned long long*>(comb_flag[i]);
  }
  a.state = state.data_ptr<int>();
  a.counts = counts.data_ptr<int>();
  a.rank = (int)rank;
  a.world = (int)W;
  a.experts_local = (int)experts_local;
  a.topk = (int)topk;
  a.cap = (int)cap;
  a.hidden = (int)hidden;
  return a;
}

#define LF_A2A_ARGS                                                                                          \
  std::vector<int64_t> recv_x, std::vector<int64_t> recv_meta, std::vector<int64_t> recv_flag,             \
      std::vector<int64_t> comb_y, std::vector<int64_t> comb_flag, const at::Tensor &state,                 \
      const at::Tensor &counts, int64_t rank, int64_t experts_local, int64_t topk, int64_t cap, int64_t hidden
#define LF_A2A_MAKE \
  make_a2a(recv_x, recv_meta, recv_flag, comb_y, comb_flag, state, counts, rank, experts_local, topk, cap, hidden)

void moe_a2a_dispatch(const at::Tensor& h, const at::Tensor& ids, at::Tensor& slot, LF_A2A_ARGS) {
  LF_CHECK(h.scalar_type() == at::kBFloat16 && h.is_contiguous() && h.size(1) == hidden, "dispatch: h [T, H] bf16");
  LF_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous() && ids.numel() == h.size(0) * topk, "dispatch: ids");
  LF_CHECK(slot.scalar_type() == at::kInt && slot.numel() >= ids.numel(), "dispatch: slot scratch");
  c10::cuda::CUDAGuard g(h.device());
  lf::a2a::dispatch(reinterpret_cast<const __nv_bfloat16*>(h.data_ptr()), ids.data_ptr<int32_t>(), h.size(0),
                    slot.data_ptr<int32_t>(), LF_A2A_MAKE, stream());
}

void moe_a2a_receive(at::Tensor& groups, at::Tensor& perm, at::Tensor& back, at::Tensor& x, LF_A2A_ARGS) {
  LF_CHECK(groups.scalar_type() == at::kInt && groups.numel() >= experts_local + 1, "receive: groups");
  LF_CHECK(perm.scalar_type() == at::kInt && back.scalar_type() == at::kLong && back.numel() >= perm.numel(),
           "receive: perm / back");
  LF_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.size(0) >= perm.numel() && x.size(1) == hidden,
           "receive: x [rows_max, H]");
  c10::cuda::CUDAGuard g(x.device());
  const lf::a2a::Args a = LF_A2A_MAKE;
  lf::a2a::receive_plan(groups.data_ptr<int32_t>(), perm.data_ptr<int32_t>(),
                        reinterpret_cast<long long*>(back.data_ptr<int64_t>()), (int)perm.numel(), a, stream());
  lf::a2a::gather(groups.data_ptr<int32_t>(), perm.data_ptr<int32_t>(),
                  reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), (int)perm.numel(), a, stream());
}

void moe_a2a_combine(const at::Tensor& y, const at::Tensor& groups, const at::Tensor& perm, const at::Tensor& back,
                     const at::Tensor& w, at::Tensor& out, LF_A2A_ARGS) {
  LF_CHECK(y.scalar_type() == at::kBFloat16 && y.is_contiguous() && y.size(1) == hidden, "combine: y");
  LF_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous() && out.scalar_type() == at::kBFloat16 &&
               out.is_contiguous() && w.numel() == out.size(0) * topk,
           "combine: w [T, k] fp32, out [T, H] bf16");
  c10::cuda::CUDAGuard g(y.device());
  const lf::a2a::Args a = LF_A2A_MAKE;
  lf::a2a::combine_send(reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), groups.data_ptr<int32_t>(),
                        perm.data_ptr<int32_t>(), reinterpret_cast<const long long*>(back.data_ptr<int64_t>()), a,
                        stream());
  lf::a2a::combine_receive(w.data_ptr<float>(), out.size(0), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), a,
                           stream());
}

// Sequence-parallel RMSNorm with the all-gather in its epilogue (sp_gather.cu).
static lf::sp::GatherArgs make_gather(const std::vector<int64_t>& dst, const std::vector<int64_t>& flag,
                                      const at::Tensor& state, int64_t rank, int64_t rows_local) {
  LF_CHECK(!dst.empty() && dst.size() <= (size_t)lf::sp::kMaxRanks && flag.size() == dst.size(),
           "norm_gather: peer lists");
  LF_CHECK(state.is_cuda() && state.scalar_type() == at::kInt && state.numel() >= 2, "norm_gather: state");
  lf::sp::GatherArgs g{};
  for (size_t i = 0; i < dst.size(); ++i) {
    g.dst[i] = reinterpret_cast<__nv_bfloat16*>(dst[i]);
    g.flag[i] = reinterpret_cast<unsigned long long*>(flag[i]);
  }
  g.state = state.data_ptr<int>();
  g.rank = (int)rank;
  g.world = (int)dst.size();
  g.rows_local = (int)rows_local;
  return g;
}

void norm_gather(const at::Tensor& x, c10::optional<at::Tensor> residual, const at::Tensor& w, double eps,
                 std::vector<int64_t> dst, std::vector<int64_t> flag, const at::Tensor& state, int64_t rank) {
  LF_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && w.is_contiguous(), "norm_gather: bf16 rows");
  if (residual.has_value())
    LF_CHECK(residual->is_contiguous() && residual->sizes() == x.sizes(), "norm_gather: residual shape");
  const lf::sp::GatherArgs g = make_gather(dst, flag, state, rank, x.size(0));
  c10::cuda::CUDAGuard gd(x.device());
  lf::sp::norm_gather(x.data_ptr(), residual.has_value() ? residual->data_ptr() : nullptr, w.data_ptr(), (float)eps,
                      x.size(1), g, stream());
  lf::sp::gather_wait(g, stream());
}

static lf::ar::LLArgs make_ll(const std::vector<int64_t>& rs, const std::vector<int64_t>& ag, int64_t ag_mc,
                              const at::Tensor& state, int64_t rank, int64_t max_pairs) {
  LF_CHECK(!rs.empty() && rs.size() <= (size_t)lf::ar::kMaxRanks && ag.size() == rs.size(), "low-latency all-reduce: peers");
  LF_CHECK(rank >= 0 && rank < (int64_t)rs.size(), "low-latency all-reduce: rank");
  LF_CHECK(state.is_cuda() && state.scalar_type() == at::kInt && state.numel() >= 2, "low-latency all-reduce: state");
  lf::ar::LLArgs a{};
  for (size_t i = 0; i < rs.size(); ++i) {
    a.rs[i] = reinterpret_cast<uint2*>(rs[i]);
    a.ag[i] = reinterpret_cast<uint2*>(ag[i]);
  }
  a.ag_mc = reinterpret_cast<uint2*>(ag_mc);
  a.state = state.data_ptr<int>();
  a.rank = (int)rank;
  a.world = (int)rs.size();
  a.max_pairs = max_pairs;
  return a;
}

// D (bf16 [M, N]) = sum over ranks of A . B^T, low-latency protocol (decode shapes).
void gemm_allreduce_ll(const at::Tensor& A, const at::Tensor& B, at::Tensor& D, at::Tensor& ws, std::vector<int64_t> rs,
                       std::vector<int64_t> ag, int64_t ag_mc, const at::Tensor& state, int64_t rank,
                       int64_t max_pairs) {
  check_rowmajor(A, "A");
  check_rowmajor(B, "B");
  check_rowmajor(D, "D");
  LF_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16 && D.scalar_type() == at::kBFloat16,
           "gemm_allreduce_ll is bf16");
  LF_CHECK(ws.scalar_type() == at::kFloat && ws.is_cuda(), "gemm_allreduce_ll: fp32 workspace");
  const int M = A.size(0), N = B.size(0), K = A.size(1);
  LF_CHECK(D.size(0) == M && D.size(1) == N, "gemm_allreduce_ll output must be [M, N]");
  lf::ar::LLArgs ll = make_ll(rs, ag, ag_mc, state, rank, max_pairs);
  c10::cuda::CUDAGuard g(A.device());
  lf::gemm::GemmArgs a{A.data_ptr(), B.data_ptr(), D.data_ptr(), M, N, K, A.stride(0), B.stride(0), D.stride(0)};
  lf::gemm::run_allreduce_ll(a, ll, stream(), ws.data_ptr<float>(), ws.numel());
}

// D = sum over ranks of the sum of `splits` fp32 [M, N] slabs of ws (low-latency protocol).
void partials_allreduce_ll(const at::Tensor& ws, int64_t splits, at::Tensor& D, std::vector<int64_t> rs,
                           std::vector<int64_t> ag, int64_t ag_mc, const at::Tensor& state, int64_t rank,
                       int64_t max_pairs) {
  check_rowmajor(D, "D");
  LF_CHECK(ws.scalar_type() == at::kFloat && ws.is_cuda() && D.scalar_type() == at::kBFloat16,
           "partials_allreduce_ll dtypes");
  const int M = D.size(0), N = D.size(1);
  LF_CHECK(ws.numel() >= splits * M * N, "partials_allreduce_ll workspace");
  lf::ar::LLArgs ll = make_ll(rs, ag, ag_mc, state, rank, max_pairs);
  c10::cuda::CUDAGuard g(D.device());
  lf::ar::finalize_ll(ws.data_ptr<float>(), (int)splits, M, N, reinterpret_cast<__nv_bfloat16*>(D.data_ptr()),
                      D.stride(0), ll, stream());
}

void gemm_grouped(const at::Tensor& A, const at::Tensor& B, at::Tensor& D, const at::Tensor& groups,
                  int64_t num_groups, int64_t epi, int64_t align) {
  check_rowmajor(A, "A");
  check_rowmajor(D, "D");
  LF_CHECK(B.is_contiguous() && B.dim() == 3 && B.size(0) >= num_groups, "grouped B must be [groups, N, K]");
  LF_CHECK(groups.scalar_type() == at::kInt && groups.numel() >= num_groups + 1, "groups must be int32 [groups+1]");
  const int M = A.size(0), N = B.size(1), K = A.size(1);
  LF_CHECK(B.size(2) == K, "grouped K mismatch");
  LF_CHECK(D.size(0) == M && D.size(1) == (epi == 2 ? N / 2 : N), "grouped output shape");
  c10::cuda::CUDAGuard g(A.device());
  lf::gemm::GemmArgs a{A.data_ptr(), B.data_ptr(), D.data_ptr(), M, N, K, A.stride(0), K, D.stride(0)};
  LF_CHECK(align == 128 || align == 256, "grouped gemm: segments aligned to 128 or 256 rows");
  lf::gemm::run_grouped(a, groups.data_ptr<int32_t>(), (int)num_groups, (int)epi, stream(), (int)align);
}

void moe_route(const at::Tensor& h, const at::Tensor& wr, c10::optional<at::Tensor> bias, int64_t topk,
               at::Tensor& ids, at::Tensor& weights) {
  LF_CHECK(h.is_contiguous() && wr.is_contiguous() && wr.scalar_type() == at::kFloat, "route operands");
  const int E = wr.size(0);
  LF_CHECK(E == 2 || E == 4 || E == 8 || E == 16, "router supports 2/4/8/16 experts");
  LF_CHECK(topk >= 1 && topk <= 8 && topk <= E && h.size(1) % 256 == 0, "route shape");
  c10::cuda::CUDAGuard g(h.device());
  lf::moe::route(h.data_ptr(), wr.data_ptr<float>(), bias.has_value() ? bias->data_ptr<float>() : nullptr,
                 h.size(0), h.size(1), E, topk, ids.data_ptr<int32_t>(), weights.data_ptr<float>(), stream());
}

void moe_align(const at::Tensor& ids, int64_t T, int64_t topk, int64_t e0, int64_t El, at::Tensor& groups,
               at::Tensor& perm, at::Tensor& slot, int64_t align) {
  LF_CHECK(El >= 1 && El <= 64, "1..64 local experts");
  LF_CHECK(align == 128 || align == 256, "moe_align: segments aligned to 128 or 256 rows");
  c10::cuda::CUDAGuard g(ids.device());
  lf::moe::align(ids.data_ptr<int32_t>(), T, topk, e0, El, perm.numel(), groups.data_ptr<int32_t>(),
                 perm.data_ptr<int32_t>(), slot.data_ptr<int32_t>(), stream(), (int)align);
}

void moe_gather(const at::Tensor& h, const at::Tensor& perm, const at::Tensor& groups, int64_t El, int64_t topk,
                at::Tensor& out) {
  c10::cuda::CUDAGuard g(h.device());
  lf::moe::gather(h.data_ptr(), perm.data_ptr<int32_t>(), groups.data_ptr<int32_t>(), El, topk, h.size(1),
                  out.size(0), out.data_ptr(), stream());
}

void moe_combine(const at::Tensor& y, const at::Tensor& slot, const at::Tensor& w, int64_t T, int64_t topk,
                 at::Tensor& out) {
  c10::cuda::CUDAGuard g(y.device());
  lf::moe::combine(y.data_ptr(), slot.data_ptr<int32_t>(), w.data_ptr<float>(), T, topk, y.size(1), out.data_ptr(),
                   stream());
}

// All-reduce of fp32 partial slabs (sum of `splits` slabs, then the sum over
// ranks) into bf16 D, through the symmetric slot given by raw addresses.
// Result region ([M, N]) = sum over ranks of the sum of `splits` fp32 slabs of ws.
void partials_allreduce(const at::Tensor& ws, int64_t M, int64_t N, int64_t splits, int64_t local, int64_t mc,
                        std::vector<int64_t> peers, int64_t out_mc, std::vector<int64_t> out_peers, int64_t cnt_local,
                        int64_t cnt_mc, std::vector<int64_t> cnt_peers, int64_t rank, int64_t cnt_capacity,
                        int64_t trace) {
  LF_CHECK(ws.scalar_type() == at::kFloat && ws.is_cuda(), "partials_allreduce: fp32 CUDA workspace");
  LF_CHECK(ws.numel() >= splits * M * N && N % 8 == 0, "partials_allreduce workspace");
  lf::gemm::ArArgs ar =
      make_ar(local, mc, peers, out_mc, out_peers, cnt_local, cnt_mc, cnt_peers, rank, cnt_capacity, trace);
  c10::cuda::CUDAGuard g(ws.device());
  lf::gemm::partials_allreduce(ws.data_ptr<float>(), (int)M, (int)N, (int)splits, ar, stream());
}

void gemm_fp8(const at::Tensor& A, const at::Tensor& sa, const at::Tensor& B, const at::Tensor& sb, at::Tensor& D,
              int64_t epi, c10::optional<at::Tensor> ws) {
  check_rowmajor(A, "A");
  check_rowmajor(B, "B");
  check_rowmajor(D, "D");
  check_rowmajor(sa, "sa");
  LF_CHECK(A.element_size() == 1 && B.element_size() == 1, "fp8 operands must be 1-byte e4m3");
  LF_CHECK(sa.scalar_type() == at::kFloat && sb.scalar_type() == at::kFloat && sb.is_contiguous(), "fp8 scales fp32");
  const int M = A.size(0), N = B.size(0), K = A.size(1);
  LF_CHECK(B.size(1) == K && K % 128 == 0 && N % 128 == 0, "fp8 gemm: K and N multiples of 128");
  LF_CHECK(sa.size(0) >= M && sa.size(1) >= K / 128 && sb.numel() >= (int64_t)(N / 128) * (K / 128), "fp8 scales");
  LF_CHECK(D.size(0) == M && D.size(1) == (epi == 2 ? N / 2 : N), "fp8 gemm output shape");
  c10::cuda::CUDAGuard g(A.device());
  lf::fp8::Fp8Args a{A.data_ptr(), B.data_ptr(), sa.data_ptr<float>(), sa.stride(0), sb.data_ptr<float>(), D.data_ptr(),
                     M, N, K, A.stride(0), B.stride(0), D.stride(0)};
  float* w = nullptr;
  int64_t w_elems = 0;
  if (ws.has_value()) {   // all-zero fp32 split-K workspace (left all-zero)
    LF_CHECK(ws->scalar_type() == at::kFloat && ws->is_contiguous() && ws->device() == A.device(),
             "fp8 gemm workspace: contiguous fp32 on the operands' device");
    w = ws->data_ptr<float>();
    w_elems = ws->numel();
  }
  lf::fp8::run(a, (int)epi, stream(), w, w_elems);
}

void act_quant(const at::Tensor& x, at::Tensor& q, at::Tensor& s) {
  check_rowmajor(x, "x");
  LF_CHECK(x.scalar_type() == at::kBFloat16 && q.element_size() == 1 && s.scalar_type() == at::kFloat, "act_quant dtypes");
  LF_CHECK(q.is_contiguous() && q.size(0) >= x.size(0) && q.size(1) == x.size(1), "act_quant output shape");
  c10::cuda::CUDAGuard g(x.device());
  lf::fp8::act_quant(x.data_ptr(), x.stride(0), x.size(0), x.size(1), q.data_ptr(), s.data_ptr<float>(), s.stride(0),
                     stream());
}

int64_t gemm_plan_splitk(int64_t M, int64_t N, int64_t K) {
  int kb = 0;
  return lf::gemm::plan_splitk(M, N, K, &kb);
}

int64_t gemm_choose_bn(int64_t M, int64_t N, int64_t epi) { return lf::gemm::choose_bn(M, N, epi); }

// (cluster size, BN, k-blocks per CTA, M-blocks per tile) of the cluster split-K plan;
// cluster size 0 = plain tiles.
std::vector<int64_t> gemm_plan_cluster(int64_t M, int64_t N, int64_t K, int64_t epi) {
  int bn = 0, kb = 0, mb = 1;
  const int c = lf::gemm::plan_cluster(M, N, K, epi, &bn, &kb, &mb);
  return {c, bn, kb, mb};
}

void gemm_set_cluster_mb2(bool on) { lf::gemm::set_cluster_mb2(on ? 1 : 0); }

void embed(at::Tensor& ids, const at::Tensor& table, at::Tensor& out, c10::optional<at::Tensor> fwd,
           int64_t fwd_first, c10::optional<at::Tensor> prev) {
  LF_CHECK(ids.scalar_type() == at::kInt && table.scalar_type() == at::kBFloat16, "embed dtypes");
  LF_CHECK(table.is_contiguous() && out.is_contiguous() && ids.is_contiguous(), "embed needs contiguous tensors");
  LF_CHECK(table.size(1) % 8 == 0, "hidden must be a multiple of 8");
  LF_CHECK(out.size(0) >= ids.size(0), "embed output too small");
  const int32_t* f = nullptr;
  const int32_t* p = nullptr;
  int nf = 0, np = 0;
  if (fwd.has_value()) {
    LF_CHECK(prev.has_value(), "embed: forwarded rows need the previous step's tokens");
    LF_CHECK(fwd->scalar_type() == at::kInt && prev->scalar_type() == at::kInt && fwd->is_contiguous() &&
                 prev->is_contiguous(), "embed: fwd / prev int32 contiguous");
    LF_CHECK(fwd_first >= 0 && fwd_first + fwd->numel() <= ids.size(0), "embed: forwarded rows outside the step");
    f = fwd->data_ptr<int32_t>();
    p = prev->data_ptr<int32_t>();
    nf = fwd->numel();
    np = prev->numel();
  }
  c10::cuda::CUDAGuard g(table.device());
  lf::ew::embed(ids.data_ptr<int32_t>(), table.data_ptr(), out.data_ptr(), ids.size(0), table.size(1), table.size(0),
                stream(), f, (int)fwd_first, nf, p, np);
}

void rmsnorm(const at::Tensor& x, c10::optional<at::Tensor> residual, const at::Tensor& w, at::Tensor& out,
             double eps, c10::optional<at::Tensor> rows) {
  LF_CHECK(x.is_contiguous() && out.is_contiguous() && w.is_contiguous(), "rmsnorm needs contiguous tensors");
  LF_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
               out.scalar_type() == at::kBFloat16, "rmsnorm is bf16");
  const int H = x.size(-1);
  LF_CHECK(H % 8 == 0 && w.numel() == H && out.size(-1) == H, "rmsnorm hidden size");
  void* r = nullptr;
  if (residual.has_value()) {
    LF_CHECK(residual->is_contiguous() && residual->numel() == x.numel(), "residual shape");
    r = residual->data_ptr();
  }
  const int in_rows = x.numel() / H;
  int out_rows = in_rows;
  const int32_t* idx = nullptr;
  if (rows.has_value()) {
    LF_CHECK(rows->scalar_type() == at::kInt && rows->is_contiguous(), "rmsnorm rows: int32 contiguous");
    out_rows = rows->numel();
    idx = rows->data_ptr<int32_t>();
  }
  LF_CHECK(out.numel() >= (int64_t)out_rows * H, "rmsnorm output too small");
  c10::cuda::CUDAGuard g(x.device());
  lf::ew::rmsnorm(x.data_ptr(), r, w.data_ptr(), out.data_ptr(), out_rows, H, (float)eps, stream(), idx, in_rows);
}

void rope_kv_write(at::Tensor& qkv, const at::Tensor& positions, const at::Tensor& slots, const at::Tensor& cos_sin,
                   at::Tensor& kcache, at::Tensor& vcache, int64_t Hq, int64_t Hkv, int64_t page) {
  check_rowmajor(qkv, "qkv");
  LF_CHECK(qkv.scalar_type() == at::kBFloat16, "qkv must be bf16");
  LF_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous(), "cos_sin must be contiguous fp32");
  LF_CHECK(kcache.is_contiguous() && vcache.is_contiguous(), "kv cache must be contiguous");
  const int D = kcache.size(-1);
  LF_CHECK(qkv.size(1) >= (Hq + 2 * Hkv) * D, "qkv width");
  LF_CHECK(positions.size(0) >= qkv.size(0) && slots.size(0) >= qkv.size(0), "positions/slots length");
  const int64_t num_slots = kcache.numel() / (Hkv * D);
  c10::cuda::CUDAGuard g(qkv.device());
  lf::ew::rope_kv_write(qkv.data_ptr(), qkv.stride(0), positions.data_ptr<int32_t>(), slots.data_ptr<int32_t>(),
                        cos_sin.data_ptr(), kcache.data_ptr(), vcache.data_ptr(), qkv.size(0), Hq, Hkv, D, page,
                        cos_sin.size(0), num_slots, stream());
}

// QKV projection with RoPE and the paged K / V write fused into the GEMM
// epilogue.  Returns false (nothing launched) when no tile plan has whole heads
// per tile; the caller then runs the GEMM and rope_kv_write.
bool gemm_qkv_rope(const at::Tensor& A, const at::Tensor& B, at::Tensor& D, const at::Tensor& positions,
                   const at::Tensor& slots, const at::Tensor& cos_sin, at::Tensor& kcache, at::Tensor& vcache,
                   int64_t Hq, int64_t Hkv, int64_t page) {
  check_cuda(A, "A");
  check_cuda(B, "B");
  check_cuda(D, "D");
  check_rowmajor(A, "A");
  check_rowmajor(B, "B");
  check_rowmajor(D, "D");
  LF_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16 && D.scalar_type() == at::kBFloat16,
           "gemm_qkv_rope is bf16");
  LF_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous() && cos_sin.numel() % 128 == 0,
           "cos_sin must be contiguous fp32 [max_pos, 64, 2]");
  LF_CHECK(kcache.is_contiguous() && vcache.is_contiguous() && kcache.size(-1) == 128, "kv cache: head_dim 128");
  LF_CHECK(positions.scalar_type() == at::kInt && slots.scalar_type() == at::kInt, "positions / slots int32");
  const int M = A.size(0), N = B.size(0), K = A.size(1);
  LF_CHECK(A.size(1) == B.size(1) && D.size(0) == M && D.size(1) == N, "gemm_qkv_rope shapes");
  LF_CHECK(N == (Hq + 2 * Hkv) * 128, "gemm_qkv_rope: N must be (Hq + 2 Hkv) * 128");
  LF_CHECK(positions.size(0) >= M && slots.size(0) >= M, "positions/slots length");
  c10::cuda::CUDAGuard g(A.device());
  lf::gemm::GemmArgs a{A.data_ptr(), B.data_ptr(), D.data_ptr(), M, N, K, A.stride(0), B.stride(0), D.stride(0)};
  lf::gemm::RopeArgs r{positions.data_ptr<int32_t>(),
                       slots.data_ptr<int32_t>(),
                       reinterpret_cast<const float2*>(cos_sin.data_ptr()),
                       reinterpret_cast<__nv_bfloat16*>(kcache.data_ptr()),
                       reinterpret_cast<__nv_bfloat16*>(vcache.data_ptr()),
                       (int)Hq,
                       (int)Hkv,
                       (int)page,
                       (int)(cos_sin.numel() / 128),
                       kcache.numel() / (Hkv * 128)};
  return lf::gemm::run_qkv_rope(a, r, stream());
}

void swiglu(const at::Tensor& gu, at::Tensor& out) {
  LF_CHECK(gu.is_contiguous() && out.is_contiguous(), "swiglu needs contiguous tensors");
  c10::cuda::CUDAGuard g(gu.device());
  lf::ew::swiglu(gu.data_ptr(), out.data_ptr(), gu.size(0), gu.size(1) / 2, stream());
}

void argmax(const at::Tensor& logits, at::Tensor& out, c10::optional<at::Tensor> status) {
  check_rowmajor(logits, "logits");
  LF_CHECK(logits.scalar_type() == at::kFloat, "logits must be fp32");
  c10::cuda::CUDAGuard g(logits.device());
  lf::ew::argmax(logits.data_ptr<float>(), logits.stride(0), logits.size(0), logits.size(1), out.data_ptr<int32_t>(),
                 status.has_value() ? status->data_ptr<int32_t>() : nullptr, stream());
}

void argmax_keys(const at::Tensor& logits, int64_t id_offset, at::Tensor& keys) {
  check_rowmajor(logits, "logits");
  LF_CHECK(logits.scalar_type() == at::kFloat, "logits must be fp32");
  LF_CHECK(keys.scalar_type() == at::kLong && keys.numel() >= logits.size(0), "keys must be int64 [rows]");
  c10::cuda::CUDAGuard g(logits.device());
  lf::ew::argmax_keys(logits.data_ptr<float>(), logits.stride(0), logits.size(0), logits.size(1), (int)id_offset,
                      reinterpret_cast<unsigned long long*>(keys.data_ptr<int64_t>()), stream());
}

void keys_to_tokens(const at::Tensor& keys, int64_t rows, int64_t ranks, at::Tensor& out) {
  LF_CHECK(keys.scalar_type() == at::kLong && keys.is_contiguous() && keys.numel() >= rows * ranks, "keys shape");
  c10::cuda::CUDAGuard g(keys.device());
  lf::ew::keys_to_tokens(reinterpret_cast<const unsigned long long*>(keys.data_ptr<int64_t>()), rows, ranks,
                         out.data_ptr<int32_t>(), stream());
}

void sample(const at::Tensor& logits, const at::Tensor& params, at::Tensor& out, c10::optional<at::Tensor> status) {
  check_rowmajor(logits, "logits");
  LF_CHECK(logits.scalar_type() == at::kFloat, "logits must be fp32");
  LF_CHECK(params.is_contiguous() && params.nbytes() >= (size_t)logits.size(0) * sizeof(lf::ew::SampleParams),
           "sample params: one 32-byte record per row");
  c10::cuda::CUDAGuard g(logits.device());
  lf::ew::sample(logits.data_ptr<float>(), logits.stride(0), logits.size(0), logits.size(1),
                 reinterpret_cast<const lf::ew::SampleParams*>(params.data_ptr()), out.data_ptr<int32_t>(),
                 status.has_value() ? status->data_ptr<int32_t>() : nullptr, stream());
}

// Vocabulary-parallel sampling, step 1: keys [rows, kc + 1] int64 (this
// shard's kc largest keys, then a status word).
void topk_keys(const at::Tensor& logits, int64_t id_offset, int64_t kc, at::Tensor& keys) {
  check_rowmajor(logits, "logits");
  LF_CHECK(logits.scalar_type() == at::kFloat, "logits must be fp32");
  LF_CHECK(kc >= 1 && kc <= 1024, "kc in [1, 1024]");
  LF_CHECK(keys.scalar_type() == at::kLong && keys.is_contiguous() && keys.numel() >= logits.size(0) * (kc + 1),
           "keys must be int64 [rows, kc + 1]");
  c10::cuda::CUDAGuard g(logits.device());
  lf::ew::topk_keys(logits.data_ptr<float>(), logits.stride(0), logits.size(0), logits.size(1), (int)id_offset,
                    (int)kc, reinterpret_cast<unsigned long long*>(keys.data_ptr<int64_t>()), stream());
}

// Step 2: the draw over every shard's candidates (keys [ranks, rows, kc + 1]).
void sample_keys(const at::Tensor& keys, int64_t rows, int64_t ranks, int64_t kc, const at::Tensor& params,
                 at::Tensor& out, c10::optional<at::Tensor> status) {
  LF_CHECK(keys.scalar_type() == at::kLong && keys.is_contiguous() && keys.numel() >= ranks * rows * (kc + 1),
           "keys must be int64 [ranks, rows, kc + 1]");
  LF_CHECK(params.is_contiguous() && params.nbytes() >= (size_t)rows * sizeof(lf::ew::SampleParams),
           "sample params: one 32-byte record per row");
  c10::cuda::CUDAGuard g(keys.device());
  lf::ew::sample_keys(reinterpret_cast<const unsigned long long*>(keys.data_ptr<int64_t>()), rows, ranks, kc,
                      reinterpret_cast<const lf::ew::SampleParams*>(params.data_ptr()), out.data_ptr<int32_t>(),
                      status.has_value() ? status->data_ptr<int32_t>() : nullptr, stream());
}

void attn_decode(const at::Tensor& q, at::Tensor& out, const at::Tensor& tok_index, const at::Tensor& seq_lens,
                 const at::Tensor& block_table, const at::Tensor& kcache, const at::Tensor& vcache, int64_t Hq,
                 int64_t Hkv, int64_t splits, c10::optional<at::Tensor> part_o, c10::optional<at::Tensor> part_lse) {
  check_rowmajor(q, "q");
  check_rowmajor(out, "out");
  check_rowmajor(block_table, "block_table");
  LF_CHECK(kcache.is_contiguous() && vcache.is_contiguous() && kcache.dim() == 4, "kv cache must be [pages, Hkv, 16, D]");
  lf::attn::DecodeArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.q_ld = q.stride(0);
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.out_ld = out.stride(0);
  a.tok_index = tok_index.data_ptr<int32_t>();
  a.seq_lens = seq_lens.data_ptr<int32_t>();
  a.block_table = block_table.data_ptr<int32_t>();
  a.bt_stride = block_table.stride(0);
  a.rows = seq_lens.size(0);
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.D = kcache.size(3);
  a.page = kcache.size(2);
  a.num_pages = kcache.size(0);
  LF_CHECK(kcache.size(1) == Hkv, "kv cache head count");
  a.splits = splits;
  a.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)a.D));
  if (splits > 1) {
    LF_CHECK(part_o.has_value() && part_lse.has_value(), "split-KV needs part_o / part_lse");
    LF_CHECK(part_o->numel() >= (int64_t)a.rows * Hq * splits * a.D && part_lse->numel() >= (int64_t)a.rows * Hq * splits,
             "split-KV workspace too small");
    a.part_o = part_o->data_ptr<float>();
    a.part_lse = part_lse->data_ptr<float>();
  }
  c10::cuda::CUDAGuard g(q.device());
  lf::attn::decode(a, kcache.data_ptr(), vcache.data_ptr(), stream());
}

int64_t attn_decode_splits(int64_t rows, int64_t Hkv, int64_t max_seq, int64_t num_sms) {
  return lf::attn::decode_splits(rows, Hkv, max_seq, num_sms);
}

void attn_prefill(const at::Tensor& q, at::Tensor& out, const at::Tensor& q_start, const at::Tensor& seq_lens,
                  const at::Tensor& block_table, const at::Tensor& kcache, const at::Tensor& vcache, int64_t Hq,
                  int64_t Hkv, int64_t max_q_len, int64_t progress) {
  check_rowmajor(q, "q");
  check_rowmajor(out, "out");
  check_rowmajor(block_table, "block_table");
  LF_CHECK(kcache.is_contiguous() && vcache.is_contiguous() && kcache.dim() == 4, "kv cache must be [pages, Hkv, 16, D]");
  lf::attn::PrefillArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.q_ld = q.stride(0);
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.out_ld = out.stride(0);
  a.q_start = q_start.data_ptr<int32_t>();
  a.seq_lens = seq_lens.data_ptr<int32_t>();
  a.block_table = block_table.data_ptr<int32_t>();
  a.bt_stride = block_table.stride(0);
  a.rows = seq_lens.size(0);
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.D = kcache.size(3);
  a.page = kcache.size(2);
  a.num_pages = kcache.size(0);
  a.max_q_len = max_q_len;
  a.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)a.D));
  a.q_rows = q.size(0);
  a.progress = reinterpret_cast<int*>(progress);
  c10::cuda::CUDAGuard g(q.device());
  lf::attn::prefill(a, kcache.data_ptr(), vcache.data_ptr(), stream());
}

std::pair<int64_t, int64_t> read_error(bool clear) {
  auto st = lf::rt::read_error(stream(), clear);
  return {st.code, (int64_t)st.info};
}

void inject_error(int64_t code) { lf::rt::inject_error((int)code); }

double counter_unit(uint64_t seed, int64_t idx) { return lf::ew::host_counter_unit(seed, idx); }

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "LunaFlux sm_100a kernels";
  m.def("gemm", &gemm, "D = A @ B^T on tcgen05 (epi 0 bf16, 1 fp32, 2 SwiGLU)", py::arg("A"), py::arg("B"),
        py::arg("D"), py::arg("epi") = 0, py::arg("bn") = 0, py::arg("ws") = py::none());
  m.def("gemm_plan_splitk", &gemm_plan_splitk);
  m.def("device_report", &lf::rt::device_report, "devices, compute capability, peer access, NVLink multicast, typed status");
  m.def("gemm_plan_cluster", &gemm_plan_cluster);
  m.def("gemm_set_cluster_mb2", &gemm_set_cluster_mb2);
  m.def("gemm_qkv_rope", &gemm_qkv_rope);
  m.def("gemm_set_pair", [](bool on) { lf::gemm::set_gemm_pair(on ? 1 : 0); });
  m.def("gemm_get_pair", []() { return lf::gemm::get_gemm_pair() != 0; });
  m.def("gemm_set_ll_fused", [](bool on) { lf::gemm::set_ll_gemm_fused(on ? 1 : 0); });
  m.def("gemm_allreduce", &gemm_allreduce);
  m.def("gemm_grouped", &gemm_grouped, py::arg("A"), py::arg("B"), py::arg("D"), py::arg("groups"),
        py::arg("num_groups"), py::arg("epi"), py::arg("align") = 128);
  m.def("gemm_fp8", &gemm_fp8, py::arg("A"), py::arg("sa"), py::arg("B"), py::arg("sb"), py::arg("D"), py::arg("epi"),
        py::arg("ws") = py::none());
  m.def("fp8_plan_splits", [](int tiles, int num_kb, int sms) {
    int per = 0;
    const int s = lf::fp8::plan_splits(tiles, num_kb, sms, &per);
    return py::make_tuple(s, per);
  });
  m.def("partials_allreduce", &partials_allreduce);
  m.def("gemm_allreduce_ll", &gemm_allreduce_ll);
  m.def("gemm_reduce_scatter", &gemm_reduce_scatter);
  m.def("norm_gather", &norm_gather);
  m.def("moe_a2a_dispatch", &moe_a2a_dispatch);
  m.def("moe_a2a_receive", &moe_a2a_receive);
  m.def("moe_a2a_combine", &moe_a2a_combine);
  m.def("partials_allreduce_ll", &partials_allreduce_ll);
  m.def("act_quant", &act_quant);
  m.def("moe_route", &moe_route);
  m.def("moe_align", &moe_align, py::arg("ids"), py::arg("T"), py::arg("topk"), py::arg("e0"), py::arg("El"),
        py::arg("groups"), py::arg("perm"), py::arg("slot"), py::arg("align") = 128);
  m.def("moe_gather", &moe_gather);
  m.def("moe_combine", &moe_combine);
  m.def("gemm_choose_bn", &gemm_choose_bn);
  m.def("embed", &embed, py::arg("ids"), py::arg("table"), py::arg("out"), py::arg("fwd") = py::none(),
        py::arg("fwd_first") = 0, py::arg("prev") = py::none());
  m.def("rmsnorm", &rmsnorm, py::arg("x"), py::arg("residual"), py::arg("w"), py::arg("out"), py::arg("eps"),
        py::arg("rows") = py::none());
  m.def("rope_kv_write", &rope_kv_write);
  m.def("swiglu", &swiglu);
  m.def("argmax", &argmax, py::arg("logits"), py::arg("out"), py::arg("status") = py::none());
  m.def("argmax_keys", &argmax_keys);
  m.def("keys_to_tokens", &keys_to_tokens);
  m.def("sample", &sample, py::arg("logits"), py::arg("params"), py::arg("out"), py::arg("status") = py::none());
  m.def("topk_keys", &topk_keys);
  m.def("sample_keys", &sample_keys, py::arg("keys"), py::arg("rows"), py::arg("ranks"), py::arg("kc"),
        py::arg("params"), py::arg("out"), py::arg("status") = py::none());
  m.def("attn_decode", &attn_decode);
  m.def("attn_decode_splits", &attn_decode_splits);
  m.def("attn_prefill", &attn_prefill, py::arg("q"), py::arg("out"), py::arg("q_start"), py::arg("seq_lens"),
        py::arg("block_table"), py::arg("kcache"), py::arg("vcache"), py::arg("Hq"), py::arg("Hkv"),
        py::arg("max_q_len"), py::arg("progress") = 0);
  m.def("read_error", &read_error, py::arg("clear") = true);
  m.def("inject_error", &inject_error);
  m.def("set_wait_limit_ns", [](int64_t ns) {
    LF_CHECK(ns > 0, "set_wait_limit_ns: the limit must be positive");
    lf::rt::set_wait_limit_ns((unsigned long long)ns);
  });
  // programmatic dependent launch of the step kernels (off by default; LUNAFLUX_PDL=1)
  m.def("set_pdl", [](bool on) { lf::rt::set_pdl(on); });
  m.def("pdl_enabled", []() { return lf::rt::pdl_enabled(); });
  m.def("counter_unit", &counter_unit);
}
