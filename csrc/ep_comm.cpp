// Native expert-parallel communicator: a symmetric device heap shared over CUDA IPC and
// the launch wrappers of the dispatch/combine kernels (moe_ep.cu).
//
// Every rank allocates one heap of identical size and layout with cudaMalloc, exports
// its IPC handle, and maps every peer's heap (cudaIpcOpenMemHandle). Kernels then store
// straight into peer memory over NVLink. The handle exchange itself is done by the
// Python caller over torch.distributed (any backend), so this class has no dependency on
// a particular bootstrap.
//
// Reference parity: replaces the NCCL all_to_all_single calls of src/rbd.py:71-133 (and
// the plan metadata exchanges of src/rbd.py:271-297) with peer stores + epoch headers.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <tuple>

#include <algorithm>
#include <string>
#include <vector>

#include "kernels.h"

namespace {

#define CUDA_OK(expr)                                                                     \
  do {                                                                                    \
    cudaError_t _e = (expr);                                                              \
    TORCH_CHECK(_e == cudaSuccess, #expr " failed: ", cudaGetErrorString(_e));            \
  } while (0)

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

class EpComm {
 public:
  EpComm(int world, int rank, int cap, int k, int hidden, int device)
      : world_(world), rank_(rank), device_(device) {
    TORCH_CHECK(world >= 1 && world <= 64, "EP world size must be in [1, 64]");
    TORCH_CHECK(rank >= 0 && rank < world, "bad rank");
    TORCH_CHECK(hidden % 8 == 0, "hidden size must be a multiple of 8");
    TORCH_CHECK(k >= 1 && k <= 8, "top-k must be in [1, 8]");
    c10::cuda::CUDAGuard g(device);
    size_t off = 0;
    auto take = [&](size_t bytes) {
      size_t o = off;
      off = align_up(off + bytes, 256);
      return o;
    };
    args_.W = world;
    args_.rank = rank;
    args_.cap = cap;
    args_.k = k;
    args_.H = hidden;
    args_.off_hdr = take(sizeof(uint64_t) * 4 * world);
    args_.off_recv_e = take(sizeof(int16_t) * (size_t)world * cap * k);
    args_.off_recv_w = take(sizeof(float) * (size_t)world * cap * k);
    args_.off_ret_w = take(sizeof(float) * (size_t)world * cap * k);
    args_.off_recv_x = take((size_t)2 * world * cap * hidden);
    args_.off_ret_x = take((size_t)2 * world * cap * hidden);
    if (hidden % 128 == 0) {  // e4m3 payload slabs for fp8 dispatch
      args_.off_recv_q = take((size_t)world * cap * hidden);
      args_.off_recv_s = take(sizeof(float) * (size_t)world * cap * (hidden / 128));
    }
    bytes_ = off;
    CUDA_OK(cudaMalloc(&heap_, bytes_));
    CUDA_OK(cudaMemset(heap_, 0, bytes_));
    for (int i = 0; i < 64; ++i) args_.peer_base[i] = nullptr;
    args_.peer_base[rank] = heap_;
  }

  ~EpComm() { close(); }

  void close() {
    if (!heap_) return;
    c10::cuda::CUDAGuard g(device_);
    cudaDeviceSynchronize();
    for (int r = 0; r < world_; ++r)
      if (r != rank_ && args_.peer_base[r]) cudaIpcCloseMemHandle(args_.peer_base[r]);
    cudaFree(heap_);
    heap_ = nullptr;
  }

  size_t heap_bytes() const { return bytes_; }

  py::bytes ipc_handle() const {
    cudaIpcMemHandle_t h;
    CUDA_OK(cudaIpcGetMemHandle(&h, heap_));
    return py::bytes(reinterpret_cast<const char*>(&h), sizeof(h));
  }

  void open_peers(const std::vector<py::bytes>& handles) {
    TORCH_CHECK((int)handles.size() == world_, "need one handle per rank");
    c10::cuda::CUDAGuard g(device_);
    for (int r = 0; r < world_; ++r) {
      if (r == rank_) continue;
      std::string s = handles[r];
      TORCH_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
      cudaIpcMemHandle_t h;
      memcpy(&h, s.data(), sizeof(h));
      void* p = nullptr;
      CUDA_OK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
      args_.peer_base[r] = p;
    }
  }

  int64_t peer_base(int r) const { return reinterpret_cast<int64_t>(args_.peer_base[r]); }

  // Graph replay: kernels add this device counter (int32, bumped once per layer call by
  // the captured sequence) to the host epoch. None restores host-only epochs.
  void set_device_epoch(const c10::optional<at::Tensor>& counter) {
    if (counter.has_value()) {
      TORCH_CHECK(counter->is_cuda() && counter->scalar_type() == at::kInt && counter->numel() == 1,
                  "device epoch counter must be one int32 on the GPU");
      epoch_dev_ = reinterpret_cast<const uint32_t*>(counter->data_ptr<int>());
    } else {
      epoch_dev_ = nullptr;
    }
  }

  // -------------------------------------------------------------------------------
  sepx::EpArgs call_args(int T, int phase, int64_t epoch, at::Tensor& done, at::Tensor& status,
                         double timeout_s) const {
    sepx::EpArgs a = args_;
    TORCH_CHECK(T <= a.cap, "more tokens than the communicator capacity");
    a.T = T;
    a.phase = phase;
    a.epoch = (uint32_t)epoch;
    a.epoch_dev = epoch_dev_;
    a.done_counter = reinterpret_cast<unsigned int*>(done.data_ptr<int>());
    a.status = status.data_ptr<int>();
    a.timeout_ns = (unsigned long long)(timeout_s * 1e9);
    return a;
  }

  void route_tables(const at::Tensor& topk_e, const at::Tensor& e2r, const at::Tensor& e2l, at::Tensor& dst,
                    at::Tensor& meta) {
    TORCH_CHECK(topk_e.scalar_type() == at::kInt && topk_e.is_contiguous(), "topk_e must be contiguous int32");
    cudaStream_t st = at::cuda::getCurrentCUDAStream().stream();
    sepx::ep_route_tables(topk_e.data_ptr<int>(), e2r.data_ptr<int>(), e2l.data_ptr<int>(), (int)topk_e.numel(),
                          dst.data_ptr<int>(), meta.data_ptr<int>(), st);
  }

  void route_plan(const at::Tensor& dst_tk, at::Tensor& slot, at::Tensor& send_count) {
    TORCH_CHECK(dst_tk.scalar_type() == at::kInt && dst_tk.is_contiguous() && dst_tk.dim() == 2, "dst_tk [T, k] int32");
    cudaStream_t st = at::cuda::getCurrentCUDAStream().stream();
    sepx::ep_route_plan(dst_tk.data_ptr<int>(), dst_tk.size(0), dst_tk.size(1), world_, slot.data_ptr<int>(),
                        send_count.data_ptr<int>(), st);
  }

  void dispatch(const at::Tensor& x, const at::Tensor& dst_tk, const at::Tensor& meta_tk, const at::Tensor& topk_w,
                const at::Tensor& slot, at::Tensor& self_tok, const at::Tensor& send_count, bool with_meta,
                int64_t epoch, at::Tensor& done, at::Tensor& status, double timeout_s, bool fp8) {
    TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "x must be contiguous bf16");
    TORCH_CHECK(x.size(1) == args_.H, "hidden size mismatch");
    TORCH_CHECK(dst_tk.size(0) == x.size(0) && meta_tk.size(0) == x.size(0), "routing rows must match tokens");
    auto a = call_args(x.size(0), 0, epoch, done, status, timeout_s);
    cudaStream_t st = at::cuda::getCurrentCUDAStream().stream();
    sepx::ep_dispatch(a, x.data_ptr(), dst_tk.data_ptr<int>(), meta_tk.data_ptr<int>(), topk_w.data_ptr<float>(),
                      slot.data_ptr<int>(), self_tok.data_ptr<int>(), send_count.data_ptr<int>(), with_meta, st, fp8);
  }

  void recv_count_scan(const at::Tensor& dst_tk, const at::Tensor& meta_tk, const at::Tensor& topk_w,
                       const at::Tensor& self_tok, const at::Tensor& send_count, int G, int T, int cap_rows,
                       int64_t epoch, at::Tensor& rows_from, at::Tensor& chunk_cnt, at::Tensor& group_off,
                       at::Tensor& group_cnt, at::Tensor& pad_off, at::Tensor& done, at::Tensor& status,
                       double timeout_s, const c10::optional<at::Tensor>& need,
                       const c10::optional<at::Tensor>& miss) {
    auto a = call_args(T, 0, epoch, done, status, timeout_s);
    cudaStream_t st = at::cuda::getCurrentCUDAStream().stream();
    int* need_p = need.has_value() ? need->data_ptr<int>() : nullptr;
    int* miss_p = miss.has_value() ? miss->data_ptr<int>() : nullptr;
    sepx::ep_recv_count_scan(a, dst_tk.data_ptr<int>(), meta_tk.data_ptr<int>(), topk_w.data_ptr<float>(),
                             self_tok.data_ptr<int>(), send_count.data_ptr<int>(), G, cap_rows,
                             rows_from.data_ptr<int>(), chunk_cnt.data_ptr<int>(), group_off.data_ptr<int>(),
                             group_cnt.data_ptr<int>(), pad_off.data_ptr<int>(), st, need_p, miss_p);
  }

  void recv_permute_gather(const at::Tensor& x, const at::Tensor& dst_tk, const at::Tensor& meta_tk,
                           const at::Tensor& topk_w, const at::Tensor& self_tok, const at::Tensor& send_count, int G,
                           int64_t epoch, const at::Tensor& rows_from, const at::Tensor& chunk_cnt,
                           const at::Tensor& group_off, const at::Tensor& group_cnt, const at::Tensor& pad_off,
                           at::Tensor& xp, at::Tensor& row_w, at::Tensor& row_src, at::Tensor& inv_rows,
                           at::Tensor& done, at::Tensor& status, double timeout_s, bool fp8) {
    TORCH_CHECK(xp.size(1) == args_.H && xp.is_contiguous(), "xp must be [rows, H]");
    auto a = call_args(x.size(0), 0, epoch, done, status, timeout_s);
    cudaStream_t st = at::cuda::getCurrentCUDAStream().stream();
    sepx::ep_recv_permute_gather(a, x.data_ptr(), dst_tk.data_ptr<int>(), meta_tk.data_ptr<int>(),
                                 topk_w.data_ptr<float>(), self_tok.data_ptr<int>(), send_count.data_ptr<int>(), G,
                                 rows_from.data_ptr<int>(), chunk_cnt.data_ptr<int>(), group_off.data_ptr<int>(),
                                 group_cnt.data_ptr<int>(), pad_off.data_ptr<int>(), xp.data_ptr(),
                                 row_w.data_ptr<float>(), row_src.data_ptr<int>(), inv_rows.data_ptr<int>(), st, fp8);
  }

  void recv_gather(const at::Tensor& x, const at::Tensor& self_tok, const at::Tensor& row_src,
                   const at::Tensor& group_off, const at::Tensor& send_count, at::Tensor& xp, int64_t epoch,
                   at::Tensor& done, at::Tensor& status, double timeout_s) {
    auto a = call_args(x.size(0), 0, epoch, done, status, timeout_s);
    cudaStream_t st = at::cuda::getCurrentCUDAStream().stream();
    const int G = group_off.size(0) - 1;
    sepx::ep_recv_gather(a, x.data_ptr(), self_tok.data_ptr<int>(), row_src.data_ptr<int>(),
                         group_off.data_ptr<int>() + G, send_count.data_ptr<int>(), xp.data_ptr(), (int)xp.size(0), st);
  }

  // The whole forward dispatch of one layer call in one host call (the per-call host cost
  // bounds a layer when nothing else keeps the GPU busy): routing tables (unless given),
  // route plan, dispatch, receive count + scan, buffer sizing, permute + gather.
  //   rows_mode > 0: the caller's row budget (need / miss record the outcome);
  //   rows_mode = 0: exact sizes (one small device->host read); rows_mode < 0: worst case.
  // Returns (tensors, rows): slot, send_count, self_tok, rows_from, group_off, group_cnt,
  // xp, row_w, row_src, inv_rows, dst_tk, meta_tk, topk_w (fp32), and the rows of xp.
  std::tuple<std::vector<at::Tensor>, int64_t> dispatch_forward(
      const at::Tensor& x, const at::Tensor& topk_e, const at::Tensor& topk_w_in, const at::Tensor& e2r,
      const at::Tensor& e2l, const c10::optional<at::Tensor>& dst_in, const c10::optional<at::Tensor>& meta_in,
      int G, int64_t epoch, int64_t rows_mode, int64_t cap_rows, const c10::optional<at::Tensor>& need,
      const c10::optional<at::Tensor>& miss, at::Tensor& done, at::Tensor& status, double timeout_s, bool fp8) {
    TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.size(1) == args_.H,
                "x must be contiguous bf16 [T, H]");
    const int64_t T = x.size(0), W = world_, k = args_.k, cap = args_.cap, H = args_.H;
    TORCH_CHECK(T <= cap, "more tokens than the communicator capacity");
    TORCH_CHECK(G >= 1 && G <= 1024, "1..1024 local expert groups");
    cudaStream_t st = at::cuda::getCurrentCUDAStream().stream();
    auto i32 = x.options().dtype(at::kInt);
    at::Tensor dst_tk, meta_tk;
    if (dst_in.has_value()) {
      dst_tk = *dst_in;
      meta_tk = *meta_in;
    } else {
      TORCH_CHECK(topk_e.scalar_type() == at::kInt && topk_e.is_contiguous(), "topk_e must be contiguous int32");
      dst_tk = at::empty({T, k}, i32);
      meta_tk = at::empty({T, k}, i32);
      sepx::ep_route_tables(topk_e.data_ptr<int>(), e2r.data_ptr<int>(), e2l.data_ptr<int>(), (int)(T * k),
                            dst_tk.data_ptr<int>(), meta_tk.data_ptr<int>(), st);
    }
    at::Tensor topk_w = topk_w_in.scalar_type() == at::kFloat && topk_w_in.is_contiguous()
                            ? topk_w_in
                            : topk_w_in.to(at::kFloat).contiguous();
    // every small int32 array of the call in one allocation
    const int64_t nchunks = W * ((cap + 127) / 128);
    const int64_t sizes[] = {T * W, W, cap, W, nchunks * G, G + 1, G, G + 1};
    int64_t total = 0;
    for (int64_t n : sizes) total += (n + 3) / 4 * 4;  // 16-byte aligned views
    at::Tensor ints = at::empty({total}, i32);
    std::vector<at::Tensor> v;
    int64_t off = 0;
    for (int64_t n : sizes) {
      v.push_back(ints.narrow(0, off, n));
      off += (n + 3) / 4 * 4;
    }
    at::Tensor slot = v[0].view({T, W}), send_count = v[1], self_tok = v[2], rows_from = v[3], chunk_cnt = v[4],
               group_off = v[5], group_cnt = v[6], pad_off = v[7];
    sepx::ep_route_plan(dst_tk.data_ptr<int>(), (int)T, (int)k, (int)W, slot.data_ptr<int>(),
                        send_count.data_ptr<int>(), st, self_tok.data_ptr<int>(), rank_);
    auto a = call_args((int)T, 0, epoch, done, status, timeout_s);
    // at world size 1 nothing is sent: the plan's self_tok is all the dispatch would write
    if (W > 1)
      sepx::ep_dispatch(a, x.data_ptr(), dst_tk.data_ptr<int>(), meta_tk.data_ptr<int>(), topk_w.data_ptr<float>(),
                        slot.data_ptr<int>(), self_tok.data_ptr<int>(), send_count.data_ptr<int>(), true, st, fp8);
    const bool budget = rows_mode > 0;
    sepx::ep_recv_count_scan(a, dst_tk.data_ptr<int>(), meta_tk.data_ptr<int>(), topk_w.data_ptr<float>(),
                             self_tok.data_ptr<int>(), send_count.data_ptr<int>(), G,
                             budget ? (int)rows_mode : (int)cap_rows, rows_from.data_ptr<int>(),
                             chunk_cnt.data_ptr<int>(), group_off.data_ptr<int>(), group_cnt.data_ptr<int>(),
                             pad_off.data_ptr<int>(), st, budget && need.has_value() ? need->data_ptr<int>() : nullptr,
                             budget && miss.has_value() ? miss->data_ptr<int>() : nullptr);
    int64_t R;
    if (rows_mode > 0) {
      R = rows_mode;
    } else if (rows_mode < 0) {
      R = cap_rows;
    } else {
      int h = 0;
      CUDA_OK(cudaMemcpyAsync(&h, group_off.data_ptr<int>() + G, sizeof(int), cudaMemcpyDeviceToHost, st));
      CUDA_OK(cudaStreamSynchronize(st));
      R = std::max<int64_t>(h, 1);
    }
    at::Tensor xp = at::empty({R, H}, x.options());
    at::Tensor row_w = at::empty({R}, x.options().dtype(at::kFloat));
    at::Tensor row_src = at::empty({R}, i32);
    at::Tensor inv_rows = at::empty({W, cap, k}, i32);
    sepx::ep_recv_permute_gather(a, x.data_ptr(), dst_tk.data_ptr<int>(), meta_tk.data_ptr<int>(),
                                 topk_w.data_ptr<float>(), self_tok.data_ptr<int>(), send_count.data_ptr<int>(), G,
                                 rows_from.data_ptr<int>(), chunk_cnt.data_ptr<int>(), group_off.data_ptr<int>(),
                                 group_cnt.data_ptr<int>(), pad_off.data_ptr<int>(), xp.data_ptr(),
                                 row_w.data_ptr<float>(), row_src.data_ptr<int>(), inv_rows.data_ptr<int>(), st, fp8);
    return {{slot, send_count, self_tok, rows_from, group_off, group_cnt, xp, row_w, row_src, inv_rows, dst_tk,
             meta_tk, topk_w},
            R};
  }

  // combine + source reduce of a forward call in one host call; returns the [T, H] output
  at::Tensor combine_forward(const at::Tensor& y, const at::Tensor& inv_rows, const at::Tensor& row_w,
                             const at::Tensor& rows_from, const at::Tensor& slot, const at::Tensor& dst_tk,
                             const c10::optional<at::Tensor>& residual, int64_t T, int64_t epoch, at::Tensor& done,
                             at::Tensor& status, double timeout_s) {
    cudaStream_t st = at::cuda::getCurrentCUDAStream().stream();
    at::Tensor out = at::empty({T, (int64_t)args_.H}, y.options());
    auto a = call_args((int)T, 1, epoch, done, status, timeout_s);
    if (world_ == 1) {  // every expert row is local: one kernel, no return slab
      sepx::ep_combine_local(a, y.data_ptr(), inv_rows.data_ptr<int>(), row_w.data_ptr<float>(),
                             slot.data_ptr<int>(), dst_tk.data_ptr<int>(), true, nullptr,
                             residual.has_value() ? residual->data_ptr() : nullptr, out.data_ptr(), nullptr, st);
      return out;
    }
    sepx::ep_combine(a, y.data_ptr(), inv_rows.data_ptr<int>(), row_w.data_ptr<float>(), rows_from.data_ptr<int>(),
                     true, nullptr, st);
    sepx::ep_source_reduce(a, slot.data_ptr<int>(), dst_tk.data_ptr<int>(),
                           residual.has_value() ? residual->data_ptr() : nullptr, out.data_ptr(), nullptr, st);
    return out;
  }

  void wait_rows(const at::Tensor& send_count, at::Tensor& rows_from, int T, int phase, int64_t epoch,
                 at::Tensor& done, at::Tensor& status, double timeout_s) {
    auto a = call_args(T, phase, epoch, done, status, timeout_s);
    cudaStream_t st = at::cuda::getCurrentCUDAStream().stream();
    sepx::ep_wait_rows(a, send_count.data_ptr<int>(), rows_from.data_ptr<int>(), st);
  }

  // Views of this rank's receive slabs (no copy): rows [W, cap, H] bf16, choice metadata
  // [W, cap, k] int16, gate weights [W, cap, k] fp32.
  std::vector<at::Tensor> slabs() const {
    auto opt = torch::TensorOptions().device(torch::kCUDA, device_);
    char* b = static_cast<char*>(heap_);
    const int64_t W = world_, cap = args_.cap, H = args_.H, k = args_.k;
    return {torch::from_blob(b + args_.off_recv_x, {W, cap, H}, opt.dtype(torch::kBFloat16)),
            torch::from_blob(b + args_.off_recv_e, {W, cap, k}, opt.dtype(torch::kShort)),
            torch::from_blob(b + args_.off_recv_w, {W, cap, k}, opt.dtype(torch::kFloat))};
  }

  void combine(const at::Tensor& y, const at::Tensor& inv_rows, const at::Tensor& row_w, const at::Tensor& rows_from,
               bool weighted, const c10::optional<at::Tensor>& row_val, int T, int64_t epoch, at::Tensor& done,
               at::Tensor& status, double timeout_s) {
    auto a = call_args(T, 1, epoch, done, status, timeout_s);
    cudaStream_t st = at::cuda::getCurrentCUDAStream().stream();
    sepx::ep_combine(a, y.data_ptr(), inv_rows.data_ptr<int>(), row_w.data_ptr<float>(), rows_from.data_ptr<int>(),
                     weighted, row_val.has_value() ? row_val->data_ptr<float>() : nullptr, st);
  }

  // World size 1: combine + source reduce in one kernel into out [T, H] (and the
  // per-choice values into val [T, k]); the same bits as combine followed by source_reduce.
  void combine_local(const at::Tensor& y, const at::Tensor& inv_rows, const at::Tensor& row_w,
                     const at::Tensor& slot, const at::Tensor& dst_tk, bool weighted,
                     const c10::optional<at::Tensor>& row_val, const c10::optional<at::Tensor>& residual,
                     at::Tensor& out, const c10::optional<at::Tensor>& val, at::Tensor& status) {
    TORCH_CHECK(world_ == 1, "combine_local runs at world size 1");
    TORCH_CHECK(out.is_contiguous() && out.size(1) == args_.H, "out must be contiguous [T, H]");
    sepx::EpArgs a = args_;
    a.T = (int)out.size(0);
    a.status = status.data_ptr<int>();
    cudaStream_t st = at::cuda::getCurrentCUDAStream().stream();
    sepx::ep_combine_local(a, y.data_ptr(), inv_rows.data_ptr<int>(), row_w.data_ptr<float>(), slot.data_ptr<int>(),
                           dst_tk.data_ptr<int>(), weighted, row_val.has_value() ? row_val->data_ptr<float>() : nullptr,
                           residual.has_value() ? residual->data_ptr() : nullptr, out.data_ptr(),
                           val.has_value() ? val->data_ptr<float>() : nullptr, st);
  }

  void source_reduce(const at::Tensor& slot, const at::Tensor& dst_tk, const c10::optional<at::Tensor>& residual,
                     at::Tensor& out, const c10::optional<at::Tensor>& val, int64_t epoch, at::Tensor& done,
                     at::Tensor& status, double timeout_s) {
    auto a = call_args(out.size(0), 1, epoch, done, status, timeout_s);
    cudaStream_t st = at::cuda::getCurrentCUDAStream().stream();
    sepx::ep_source_reduce(a, slot.data_ptr<int>(), dst_tk.data_ptr<int>(),
                           residual.has_value() ? residual->data_ptr() : nullptr, out.data_ptr(),
                           val.has_value() ? val->data_ptr<float>() : nullptr, st);
  }

 private:
  int world_, rank_, device_;
  void* heap_ = nullptr;
  size_t bytes_ = 0;
  sepx::EpArgs args_;
  const uint32_t* epoch_dev_ = nullptr;
};

// Generic symmetric buffer: one cudaMalloc per rank, IPC-mapped on every peer. ``put``
// copies a local tensor into a peer's buffer with one cudaMemcpyAsync (copy engine over
// NVLink); used by the expert-weight transfer path (placement changes) and its benchmark.
class SymmBuffer {
 public:
  SymmBuffer(int world, int rank, int64_t bytes, int device) : world_(world), rank_(rank), device_(device) {
    TORCH_CHECK(world >= 1 && world <= 64 && rank >= 0 && rank < world, "bad world/rank");
    c10::cuda::CUDAGuard g(device);
    bytes_ = (size_t)bytes;
    CUDA_OK(cudaMalloc(&base_, bytes_));
    CUDA_OK(cudaMemset(base_, 0, bytes_));
    peers_.assign(world, nullptr);
    peers_[rank] = base_;
  }
  ~SymmBuffer() { close(); }
  void close() {
    if (!base_) return;
    c10::cuda::CUDAGuard g(device_);
    cudaDeviceSynchronize();
    for (int r = 0; r < world_; ++r)
      if (r != rank_ && peers_[r]) cudaIpcCloseMemHandle(peers_[r]);
    cudaFree(base_);
    base_ = nullptr;
  }
  py::bytes ipc_handle() const {
    cudaIpcMemHandle_t h;
    CUDA_OK(cudaIpcGetMemHandle(&h, base_));
    return py::bytes(reinterpret_cast<const char*>(&h), sizeof(h));
  }
  void open_peers(const std::vector<py::bytes>& handles) {
    TORCH_CHECK((int)handles.size() == world_, "need one handle per rank");
    c10::cuda::CUDAGuard g(device_);
    for (int r = 0; r < world_; ++r) {
      if (r == rank_) continue;
      std::string s = handles[r];
      cudaIpcMemHandle_t h;
      memcpy(&h, s.data(), sizeof(h));
      CUDA_OK(cudaIpcOpenMemHandle(&peers_[r], h, cudaIpcMemLazyEnablePeerAccess));
    }
  }
  // local view as a uint8 tensor (no copy; lifetime tied to this object)
  at::Tensor local() const {
    return torch::from_blob(base_, {(int64_t)bytes_}, torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device_));
  }
  void put(const at::Tensor& src, int peer, int64_t byte_offset) {
    TORCH_CHECK(src.is_cuda() && src.is_contiguous(), "src must be a contiguous CUDA tensor");
    TORCH_CHECK(peer >= 0 && peer < world_ && peers_[peer], "peer not mapped");
    const size_t n = src.numel() * src.element_size();
    TORCH_CHECK(byte_offset >= 0 && (size_t)byte_offset + n <= bytes_, "put out of bounds");
    cudaStream_t st = at::cuda::getCurrentCUDAStream().stream();
    CUDA_OK(cudaMemcpyAsync(static_cast<char*>(peers_[peer]) + byte_offset, src.data_ptr(), n,
                            cudaMemcpyDeviceToDevice, st));
  }
  int64_t size() const { return (int64_t)bytes_; }

  // All-to-all write bandwidth probe: this rank writes `bytes_per_peer` of src into every
  // other rank's buffer at offset rank * bytes_per_peer (mode 0: SM stores, 1: TMA bulk).
  void p2p_write_bench(const at::Tensor& src, int64_t bytes_per_peer, int mode, int blocks,
                       const at::Tensor& status) {
    TORCH_CHECK(src.is_cuda() && src.is_contiguous() && src.numel() * src.element_size() >= bytes_per_peer,
                "src must hold bytes_per_peer bytes");
    TORCH_CHECK((int64_t)bytes_ >= bytes_per_peer * world_, "buffer too small");
    sepx::P2PBenchArgs a;
    for (int r = 0; r < 64; ++r) a.dst[r] = r < world_ ? static_cast<uint8_t*>(peers_[r]) : nullptr;
    a.src = static_cast<const uint8_t*>(src.data_ptr());
    a.bytes_per_peer = bytes_per_peer;
    a.W = world_;
    a.rank = rank_;
    a.mode = mode;
    a.status = status.data_ptr<int>();
    sepx::p2p_write_bench(a, blocks, at::cuda::getCurrentCUDAStream().stream());
  }

  // Speculative replication: copy the experts named by (fetch_rank[s], fetch_slot[s])
  // from their primary rank's buffer into local cache slot P + s of every region
  // (region r holds [slots][reg_stride[r] bytes] at byte reg_off[r]). One kernel with
  // plain peer loads; the slot choice stays on the device.
  void fetch_experts(int P, int src_limit, const std::vector<int64_t>& reg_off,
                     const std::vector<int64_t>& reg_stride, const at::Tensor& fetch_rank,
                     const at::Tensor& fetch_slot, int blocks_per_slot) {
    TORCH_CHECK(reg_off.size() == reg_stride.size() && !reg_off.empty() && reg_off.size() <= 4,
                "1 to 4 weight regions");
    TORCH_CHECK(fetch_rank.is_cuda() && fetch_rank.scalar_type() == at::kInt && fetch_rank.is_contiguous(),
                "fetch_rank must be a contiguous int32 CUDA tensor");
    TORCH_CHECK(fetch_slot.is_cuda() && fetch_slot.scalar_type() == at::kInt && fetch_slot.is_contiguous() &&
                    fetch_slot.numel() == fetch_rank.numel(),
                "fetch_slot must match fetch_rank");
    const int S = (int)fetch_rank.numel();
    TORCH_CHECK(P >= 1 && S >= 1, "need primary and cache slots");
    TORCH_CHECK(src_limit >= 1, "src_limit must be positive");
    for (int r = 0; r < world_; ++r) TORCH_CHECK(peers_[r], "peer ", r, " not mapped");
    sepx::SpecFetchArgs a;
    for (int r = 0; r < 64; ++r) a.peer_base[r] = r < world_ ? peers_[r] : nullptr;
    a.local_base = base_;
    a.W = world_;
    a.P = P;
    a.S = S;
    a.src_limit = src_limit;
    a.nreg = (int)reg_off.size();
    // every rank's buffer has the same size and layout, so bounds checked here hold on peers
    const size_t slots = (size_t)std::max(P + S, src_limit);
    for (int r = 0; r < a.nreg; ++r) {
      TORCH_CHECK(reg_off[r] >= 0 && reg_stride[r] > 0 && (size_t)reg_off[r] + slots * (size_t)reg_stride[r] <= bytes_,
                  "weight region ", r, " does not fit the buffer");
      a.reg_off[r] = (size_t)reg_off[r];
      a.reg_stride[r] = (size_t)reg_stride[r];
    }
    a.fetch_rank = fetch_rank.data_ptr<int>();
    a.fetch_slot = fetch_slot.data_ptr<int>();
    c10::cuda::CUDAGuard g(device_);
    sepx::spec_fetch(a, blocks_per_slot, at::cuda::getCurrentCUDAStream().stream());
  }

 private:
  int world_, rank_, device_;
  void* base_ = nullptr;
  size_t bytes_ = 0;
  std::vector<void*> peers_;
};

// Speculative replication policy: one block turns predicted expert ids into cache
// updates, fetch orders and routing tables (speculative.cu).
void spec_policy(const at::Tensor& pred_e, int rank, int P, int min_count, const at::Tensor& base_e2r,
                 const at::Tensor& base_e2l, const at::Tensor& owner, const at::Tensor& owner_slot,
                 at::Tensor& slot_expert, at::Tensor& slot_stamp, at::Tensor& step, at::Tensor& e2r, at::Tensor& e2l,
                 at::Tensor& fetch_rank, at::Tensor& fetch_slot, const c10::optional<at::Tensor>& stats) {
  auto ok = [](const at::Tensor& t, const char* name) {
    TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kInt && t.is_contiguous(), name,
                " must be a contiguous int32 CUDA tensor");
  };
  ok(pred_e, "pred_e");
  ok(base_e2r, "base_e2r");
  ok(base_e2l, "base_e2l");
  ok(owner, "owner");
  ok(owner_slot, "owner_slot");
  ok(slot_expert, "slot_expert");
  ok(slot_stamp, "slot_stamp");
  ok(step, "step");
  ok(e2r, "e2r");
  ok(e2l, "e2l");
  ok(fetch_rank, "fetch_rank");
  ok(fetch_slot, "fetch_slot");
  TORCH_CHECK(pred_e.dim() == 2, "pred_e must be [T, k]");
  const int E = (int)base_e2r.numel(), S = (int)slot_expert.numel();
  TORCH_CHECK(base_e2l.numel() == E && owner.numel() == E && owner_slot.numel() == E && e2r.numel() == E &&
                  e2l.numel() == E,
              "expert tables must all have E entries");
  TORCH_CHECK(slot_stamp.numel() == S && fetch_rank.numel() == S && fetch_slot.numel() == S && step.numel() == 1,
              "cache tensors must all have S entries");
  sepx::SpecPolicyArgs a;
  a.pred_e = pred_e.data_ptr<int>();
  a.T = (int)pred_e.size(0);
  a.k = (int)pred_e.size(1);
  a.E = E;
  a.S = S;
  a.P = P;
  a.rank = rank;
  a.min_count = min_count;
  a.base_e2r = base_e2r.data_ptr<int>();
  a.base_e2l = base_e2l.data_ptr<int>();
  a.owner = owner.data_ptr<int>();
  a.owner_slot = owner_slot.data_ptr<int>();
  a.slot_expert = slot_expert.data_ptr<int>();
  a.slot_stamp = slot_stamp.data_ptr<int>();
  a.step = step.data_ptr<int>();
  a.e2r = e2r.data_ptr<int>();
  a.e2l = e2l.data_ptr<int>();
  a.fetch_rank = fetch_rank.data_ptr<int>();
  a.fetch_slot = fetch_slot.data_ptr<int>();
  if (stats.has_value()) {
    TORCH_CHECK(stats->is_cuda() && stats->scalar_type() == at::kLong && stats->numel() == 4,
                "stats must be 4 int64 on the GPU");
    a.stats = reinterpret_cast<long long*>(stats->data_ptr<int64_t>());
  }
  c10::cuda::CUDAGuard g(pred_e.device());
  sepx::spec_policy(a, at::cuda::getCurrentCUDAStream().stream());
}

}  // namespace

void register_ep_comm(pybind11::module& m) {
  m.def("spec_policy", &spec_policy, "speculative replica cache update (LRU) + routing tables");
  py::class_<EpComm>(m, "EpComm")
      .def(py::init<int, int, int, int, int, int>(), py::arg("world"), py::arg("rank"), py::arg("cap"),
           py::arg("k"), py::arg("hidden"), py::arg("device"))
      .def("close", &EpComm::close)
      .def("heap_bytes", &EpComm::heap_bytes)
      .def("ipc_handle", &EpComm::ipc_handle)
      .def("open_peers", &EpComm::open_peers)
      .def("peer_base", &EpComm::peer_base)
      .def("set_device_epoch", &EpComm::set_device_epoch)
      .def("route_tables", &EpComm::route_tables)
      .def("route_plan", &EpComm::route_plan)
      .def("dispatch", &EpComm::dispatch)
      .def("recv_count_scan", &EpComm::recv_count_scan)
      .def("dispatch_forward", &EpComm::dispatch_forward)
      .def("combine_forward", &EpComm::combine_forward)
      .def("recv_permute_gather", &EpComm::recv_permute_gather)
      .def("recv_gather", &EpComm::recv_gather)
      .def("wait_rows", &EpComm::wait_rows)
      .def("slabs", &EpComm::slabs)
      .def("combine", &EpComm::combine)
      .def("combine_local", &EpComm::combine_local)
      .def("source_reduce", &EpComm::source_reduce);
  py::class_<SymmBuffer>(m, "SymmBuffer")
      .def(py::init<int, int, int64_t, int>(), py::arg("world"), py::arg("rank"), py::arg("bytes"), py::arg("device"))
      .def("close", &SymmBuffer::close)
      .def("ipc_handle", &SymmBuffer::ipc_handle)
      .def("open_peers", &SymmBuffer::open_peers)
      .def("local", &SymmBuffer::local)
      .def("put", &SymmBuffer::put)
      .def("fetch_experts", &SymmBuffer::fetch_experts)
      .def("p2p_write_bench", &SymmBuffer::p2p_write_bench)
      .def("size", &SymmBuffer::size);
}
