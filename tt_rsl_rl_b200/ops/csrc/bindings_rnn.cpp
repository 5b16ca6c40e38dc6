// Python bindings of the GRU / LSTM cell kernels. Every array is passed as a tensor (its first element) plus its row
// pitch in elements, so strided views of env-major [env, T, width] buffers can be used directly.
#include <torch/extension.h>

#include <utility>

#include <c10/cuda/CUDAStream.h>

#include "gemm_tcgen05.cuh"
#include "kernels.cuh"
#include "rnn_kernels.cuh"

namespace {

using torch::Tensor;
using OptT = c10::optional<Tensor>;

cudaStream_t cur() { return c10::cuda::getCurrentCUDAStream().stream(); }

int64_t avail(const Tensor& t) {
  return static_cast<int64_t>(t.storage().nbytes() / t.element_size()) - t.storage_offset();
}

// The array of `rows` rows of `width` elements at pitch ld must lie inside the tensor's storage.
template <typename T>
T* ptr(const OptT& t, int64_t rows, int64_t ld, int64_t width, c10::ScalarType dt, const char* name) {
  if (!t.has_value()) return nullptr;
  TORCH_CHECK(t->is_cuda() && t->scalar_type() == dt, name, ": wrong device or dtype");
  TORCH_CHECK(rows <= 0 || avail(*t) >= (rows - 1) * ld + width, name, ": too small for rows x width at pitch ld");
  return reinterpret_cast<T*>(t->data_ptr());
}

void ok(cudaError_t e, const char* what) { TORCH_CHECK(e == cudaSuccess, what, ": ", cudaGetErrorString(e)); }

void rnn_cell_fwd(int64_t rows, int64_t H, bool lstm, const Tensor& gi, int64_t ld_gi, const Tensor& gh, int64_t ld_gh,
                  const Tensor& h_in, int64_t ld_h_in, const OptT& c_in, int64_t ld_c_in, const OptT& h_out,
                  int64_t ld_h_out, const OptT& h_out_bf16, int64_t ld_h_out_bf16, const OptT& c_out, int64_t ld_c_out,
                  const OptT& done, const OptT& next_h, int64_t ld_next_h, const OptT& next_h_bf16,
                  int64_t ld_next_h_bf16, const OptT& next_c, int64_t ld_next_c, const OptT& save, int64_t ld_save) {
  const int64_t G = lstm ? 4 : 3, S = lstm ? 5 : 4;
  const auto f32 = torch::kFloat32, bf = torch::kBFloat16;
  rlb::RnnCellFwdArgs a{};
  a.rows = static_cast<int>(rows);
  a.H = static_cast<int>(H);
  a.lstm = lstm ? 1 : 0;
  a.gi = ptr<const float>(gi, rows, ld_gi, G * H, f32, "gi");
  a.ld_gi = ld_gi;
  a.gh = ptr<const float>(gh, rows, ld_gh, G * H, f32, "gh");
  a.ld_gh = ld_gh;
  a.h_in = ptr<const float>(h_in, rows, ld_h_in, H, f32, "h_in");
  a.ld_h_in = ld_h_in;
  a.c_in = ptr<const float>(c_in, rows, ld_c_in, H, f32, "c_in");
  a.ld_c_in = ld_c_in;
  a.h_out = ptr<float>(h_out, rows, ld_h_out, H, f32, "h_out");
  a.ld_h_out = ld_h_out;
  a.h_out_bf16 = ptr<void>(h_out_bf16, rows, ld_h_out_bf16, H, bf, "h_out_bf16");
  a.ld_h_out_bf16 = ld_h_out_bf16;
  a.c_out = ptr<float>(c_out, rows, ld_c_out, H, f32, "c_out");
  a.ld_c_out = ld_c_out;
  a.done = ptr<const float>(done, 1, 1, rows, f32, "done");
  a.next_h = ptr<float>(next_h, rows, ld_next_h, H, f32, "next_h");
  a.ld_next_h = ld_next_h;
  a.next_h_bf16 = ptr<void>(next_h_bf16, rows, ld_next_h_bf16, H, bf, "next_h_bf16");
  a.ld_next_h_bf16 = ld_next_h_bf16;
  a.next_c = ptr<float>(next_c, rows, ld_next_c, H, f32, "next_c");
  a.ld_next_c = ld_next_c;
  a.save = ptr<float>(save, rows, ld_save, S * H, f32, "save");
  a.ld_save = ld_save;
  TORCH_CHECK(!lstm || (a.c_in != nullptr && a.c_out != nullptr), "rnn_cell_fwd: LSTM needs c_in and c_out");
  ok(rlb::rnn_cell_fwd(a, cur()), "rnn_cell_fwd");
}

void rnn_cell_bwd(int64_t rows, int64_t H, bool lstm, const Tensor& save, int64_t ld_save, const OptT& h_in,
                  int64_t ld_h_in, const OptT& c_in, int64_t ld_c_in, const Tensor& dh_head, int64_t ld_dh_head,
                  const OptT& dh_rec_a, const OptT& dh_rec_b, int64_t ld_dh_rec, const OptT& dc_rec, int64_t ld_dc_rec,
                  const OptT& done, const Tensor& dgi, int64_t ld_dgi, const OptT& dgh, int64_t ld_dgh,
                  const OptT& dh_direct, int64_t ld_dh_direct, const OptT& dc_prev, int64_t ld_dc_prev,
                  const OptT& colsum_gi, const OptT& colsum_gh, bool colsum_accumulate) {
  const int64_t G = lstm ? 4 : 3, S = lstm ? 5 : 4;
  const auto f32 = torch::kFloat32, bf = torch::kBFloat16;
  const int64_t blocks = rlb::rnn_bwd_blocks(static_cast<int>(rows));
  rlb::RnnCellBwdArgs a{};
  a.rows = static_cast<int>(rows);
  a.H = static_cast<int>(H);
  a.lstm = lstm ? 1 : 0;
  a.save = ptr<const float>(save, rows, ld_save, S * H, f32, "save");
  a.ld_save = ld_save;
  a.h_in = ptr<const float>(h_in, rows, ld_h_in, H, f32, "h_in");
  a.ld_h_in = ld_h_in;
  a.c_in = ptr<const float>(c_in, rows, ld_c_in, H, f32, "c_in");
  a.ld_c_in = ld_c_in;
  a.dh_head = ptr<const float>(dh_head, rows, ld_dh_head, H, f32, "dh_head");
  a.ld_dh_head = ld_dh_head;
  a.dh_rec_a = ptr<const float>(dh_rec_a, rows, ld_dh_rec, H, f32, "dh_rec_a");
  a.dh_rec_b = ptr<const float>(dh_rec_b, rows, ld_dh_rec, H, f32, "dh_rec_b");
  a.ld_dh_rec = ld_dh_rec;
  a.dc_rec = ptr<const float>(dc_rec, rows, ld_dc_rec, H, f32, "dc_rec");
  a.ld_dc_rec = ld_dc_rec;
  a.done = ptr<const float>(done, 1, 1, rows, f32, "done");
  a.dgi = ptr<void>(dgi, rows, ld_dgi, G * H, bf, "dgi");
  a.ld_dgi = ld_dgi;
  a.dgh = ptr<void>(dgh, rows, ld_dgh, G * H, bf, "dgh");
  a.ld_dgh = ld_dgh;
  a.dh_direct = ptr<float>(dh_direct, rows, ld_dh_direct, H, f32, "dh_direct");
  a.ld_dh_direct = ld_dh_direct;
  a.dc_prev = ptr<float>(dc_prev, rows, ld_dc_prev, H, f32, "dc_prev");
  a.ld_dc_prev = ld_dc_prev;
  a.colsum_gi = ptr<float>(colsum_gi, blocks, G * H, G * H, f32, "colsum_gi");
  a.colsum_gh = ptr<float>(colsum_gh, blocks, G * H, G * H, f32, "colsum_gh");
  a.colsum_accumulate = colsum_accumulate ? 1 : 0;
  ok(rlb::rnn_cell_bwd(a, cur()), "rnn_cell_bwd");
}

void rnn_mask(int64_t rows, int64_t H, const Tensor& src_h, int64_t ld_src_h, const OptT& src_c, int64_t ld_src_c,
              const OptT& done, const OptT& dst_h, int64_t ld_dst_h, const OptT& dst_h_bf16, int64_t ld_dst_h_bf16,
              const OptT& dst_c, int64_t ld_dst_c) {
  const auto f32 = torch::kFloat32, bf = torch::kBFloat16;
  rlb::RnnMaskArgs a{};
  a.rows = static_cast<int>(rows);
  a.H = static_cast<int>(H);
  a.src_h = ptr<const float>(src_h, rows, ld_src_h, H, f32, "src_h");
  a.ld_src_h = ld_src_h;
  a.src_c = ptr<const float>(src_c, rows, ld_src_c, H, f32, "src_c");
  a.ld_src_c = ld_src_c;
  a.done = ptr<const float>(done, 1, 1, rows, f32, "done");
  a.dst_h = ptr<float>(dst_h, rows, ld_dst_h, H, f32, "dst_h");
  a.ld_dst_h = ld_dst_h;
  a.dst_h_bf16 = ptr<void>(dst_h_bf16, rows, ld_dst_h_bf16, H, bf, "dst_h_bf16");
  a.ld_dst_h_bf16 = ld_dst_h_bf16;
  a.dst_c = ptr<float>(dst_c, rows, ld_dst_c, H, f32, "dst_c");
  a.ld_dst_c = ld_dst_c;
  ok(rlb::rnn_mask(a, cur()), "rnn_mask");
}

int64_t rnn_bwd_blocks(int64_t rows) { return rlb::rnn_bwd_blocks(static_cast<int>(rows)); }

// One recurrent step in one launch: gh = h_bf16 W_hh^T on the tensor cores and the cell in the GEMM's epilogue
// (gemm_tcgen05.cuh kEpiRnnCell). Arguments as rnn_cell_fwd, with the GEMM operands in place of gh.
void rnn_step_fused(int64_t rows, int64_t H, bool lstm, const Tensor& a, int64_t ld_a, const Tensor& w_hh,
                    int64_t ld_w, const Tensor& b_hh, const Tensor& gi, int64_t ld_gi, const OptT& h_in,
                    int64_t ld_h_in, const OptT& c_in, int64_t ld_c_in, const OptT& h_out, int64_t ld_h_out,
                    const OptT& h_out_bf16, int64_t ld_h_out_bf16, const OptT& c_out, int64_t ld_c_out,
                    const OptT& done, const OptT& next_h, int64_t ld_next_h, const OptT& next_h_bf16,
                    int64_t ld_next_h_bf16, const OptT& next_c, int64_t ld_next_c, const OptT& save, int64_t ld_save,
                    const OptT& status) {
  const int64_t G = lstm ? 4 : 3, S = lstm ? 5 : 4;
  const auto f32 = torch::kFloat32, bf = torch::kBFloat16;
  TORCH_CHECK(rows > 0 && H > 0 && H % rlb::kRnnUnits == 0, "rnn_step_fused: H must be a multiple of ",
              rlb::kRnnUnits);
  rlb::GemmParams p;
  p.a = ptr<const void>(a, rows, ld_a, H, bf, "a");
  p.lda = static_cast<int>(ld_a);
  p.b = ptr<const void>(w_hh, G * H, ld_w, H, bf, "w_hh");
  p.ldb = static_cast<int>(ld_w);
  p.M = static_cast<int>(rows);
  p.N = static_cast<int>(G * H);
  p.K = static_cast<int>(H);
  p.epilogue = rlb::kEpiRnnCell;
  p.bias = ptr<const float>(b_hh, 1, 1, G * H, f32, "b_hh");
  if (status.has_value()) {
    TORCH_CHECK(status->is_cuda() && status->scalar_type() == torch::kInt32, "rnn_step_fused: status");
    p.status = reinterpret_cast<unsigned int*>(status->data_ptr());
  }
  rlb::RnnCellEpi& e = p.cell;
  e.H = static_cast<int>(H);
  e.lstm = lstm ? 1 : 0;
  e.gi = ptr<const float>(gi, rows, ld_gi, G * H, f32, "gi");
  e.ld_gi = ld_gi;
  e.h_in = ptr<const float>(h_in, rows, ld_h_in, H, f32, "h_in");
  e.ld_h_in = ld_h_in;
  e.c_in = ptr<const float>(c_in, rows, ld_c_in, H, f32, "c_in");
  e.ld_c_in = ld_c_in;
  e.h_out = ptr<float>(h_out, rows, ld_h_out, H, f32, "h_out");
  e.ld_h_out = ld_h_out;
  e.h_out_bf16 = ptr<void>(h_out_bf16, rows, ld_h_out_bf16, H, bf, "h_out_bf16");
  e.ld_h_out_bf16 = ld_h_out_bf16;
  e.c_out = ptr<float>(c_out, rows, ld_c_out, H, f32, "c_out");
  e.ld_c_out = ld_c_out;
  e.done = ptr<const float>(done, 1, 1, rows, f32, "done");
  e.next_h = ptr<float>(next_h, rows, ld_next_h, H, f32, "next_h");
  e.ld_next_h = ld_next_h;
  e.next_h_bf16 = ptr<void>(next_h_bf16, rows, ld_next_h_bf16, H, bf, "next_h_bf16");
  e.ld_next_h_bf16 = ld_next_h_bf16;
  e.next_c = ptr<float>(next_c, rows, ld_next_c, H, f32, "next_c");
  e.ld_next_c = ld_next_c;
  e.save = ptr<float>(save, rows, ld_save, S * H, f32, "save");
  e.ld_save = ld_save;
  // The A operand (all units of a row) is read by every unit tile: no bf16 output may overwrite it during the
  // launch. Outputs in the same buffer are allowed when they are other columns of the same row pitch (the next
  // step's slot of an env-major [env, T, H] buffer).
  const long long a_span = (rows - 1) * ld_a + H;
  const auto a_lo = reinterpret_cast<intptr_t>(p.a);
  const std::pair<const void*, int64_t> outs[2] = {{e.h_out_bf16, ld_h_out_bf16}, {e.next_h_bf16, ld_next_h_bf16}};
  for (const auto& [o, ld_o] : outs) {
    if (o == nullptr) continue;
    const auto o_lo = reinterpret_cast<intptr_t>(o);
    const long long o_span = (rows - 1) * ld_o + H;
    if (o_lo >= a_lo + 2 * a_span || o_lo + 2 * o_span <= a_lo) continue;  // disjoint address ranges
    const long long d = (o_lo - a_lo) / 2;
    const long long r = ((d % ld_a) + ld_a) % ld_a;
    TORCH_CHECK(ld_o == ld_a && (o_lo - a_lo) % 2 == 0 && r >= H && r <= ld_a - H,
                "rnn_step_fused: a bf16 output overlaps the input state operand");
  }
  ok(rlb::gemm_launch(p, cur()), "rnn_step_fused");
}

void rnn_pad_entries(const Tensor& done, int64_t T, int64_t N, int64_t lo, int64_t Be, const Tensor& out) {
  TORCH_CHECK(done.is_cuda() && done.scalar_type() == torch::kFloat32 && done.is_contiguous() &&
                  done.numel() >= T * N,
              "rnn_pad_entries: done must be a contiguous fp32 [T * N] CUDA tensor");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == torch::kFloat32 && out.numel() >= 1,
              "rnn_pad_entries: out must be fp32 on the device");
  ok(rlb::rnn_pad_entries(done.data_ptr<float>(), static_cast<int>(T), static_cast<int>(N), static_cast<int>(lo),
                          static_cast<int>(Be), out.data_ptr<float>(), cur()),
     "rnn_pad_entries");
}

}  // namespace

void rlb_register_rnn(pybind11::module& m) {
  m.def("rnn_cell_fwd", &rnn_cell_fwd);
  m.def("rnn_cell_bwd", &rnn_cell_bwd);
  m.def("rnn_mask", &rnn_mask);
  m.def("rnn_bwd_blocks", &rnn_bwd_blocks);
  m.def("rnn_pad_entries", &rnn_pad_entries);
  m.def("rnn_step_fused", &rnn_step_fused);
}
