// Python binding of the hot calls for torch tensors: one object per buffer
// allocates the outputs with ATen, takes the current CUDA stream and calls
// the C ABI (per_b200.h) directly. It replaces the ctypes round trip and the
// Python-level allocation and view building of sample() / update_priorities()
// (host cost per call, which bounds small-batch throughput outside CUDA
// graphs). No kernels here: everything runs in libper_b200.so.
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <string>
#include <vector>

#include "per_b200.h"

namespace py = pybind11;

namespace {

class Engine {
 public:
  Engine(int64_t store, int64_t device, std::vector<std::string> names, std::vector<int64_t> dims,
         int64_t rng_counter, int64_t row_dtype)
      : store_(reinterpret_cast<const per_store_t*>(store)),
        row_dtype_(row_dtype == 1 ? at::kBFloat16 : row_dtype == 2 ? at::kHalf : at::kFloat),
        device_(static_cast<c10::DeviceIndex>(device)),
        names_(std::move(names)),
        dims_(std::move(dims)),
        counter_(reinterpret_cast<uint64_t*>(rng_counter)) {
    row_dim_ = 0;
    for (int64_t d : dims_) row_dim_ += d;
    py_names_ = py::list();
    for (const auto& n : names_) py_names_.append(py::str(n));
  }

  // sample(batch, beta, seed) -> (rc, {name: view}, idx, w), uniforms drawn in the kernel
  py::tuple sample(int64_t batch, double beta, uint64_t seed) {
    c10::cuda::CUDAGuard guard(device_);
    at::Tensor out, idx, w;
    alloc(batch, &out, &idx, &w);
    const int rc = per_sample_fused_rng(store_, seed, counter_, batch, static_cast<float>(beta),
                                        rows(out), row_dim_, idx.data_ptr<int64_t>(),
                                        w.data_ptr<float>(), stream());
    return py::make_tuple(rc, views(out), idx, w);
  }

  // sample(batch, beta, seed) into caller-owned device buffers -> rc: rows
  // (row_stride elements apart), idx (int64) and w (float32), checked by the
  // caller once when the destination was made; nothing allocated, no views
  int sample_into(int64_t batch, double beta, uint64_t seed, int64_t rows, int64_t row_stride,
                  int64_t idx, int64_t w) {
    c10::cuda::CUDAGuard guard(device_);
    return per_sample_fused_rng(store_, seed, counter_, batch, static_cast<float>(beta),
                                reinterpret_cast<float*>(rows), row_stride,
                                reinterpret_cast<int64_t*>(idx), reinterpret_cast<float*>(w),
                                stream());
  }

  // sample_from(rand, beta) -> (rc, views, idx, w) with caller uniforms (float32, contiguous)
  py::tuple sample_from(const at::Tensor& rand, double beta) {
    c10::cuda::CUDAGuard guard(device_);
    const int64_t batch = rand.numel();
    at::Tensor out, idx, w;
    alloc(batch, &out, &idx, &w);
    const int rc = per_sample_fused(store_, rand.data_ptr<float>(), batch, static_cast<float>(beta),
                                    rows(out), row_dim_, idx.data_ptr<int64_t>(),
                                    w.data_ptr<float>(), stream());
    return py::make_tuple(rc, views(out), idx, w);
  }

  // sharded sample with the in-kernel exchange and uniforms:
  // -> (rc, views, idx, w, pos, count) of this rank's owned draws
  // local: weights normalised by this rank's own max (no max exchange)
  py::tuple sample_sharded_p2p(int32_t rank, int32_t world, int64_t shard_base, int64_t mailboxes,
                               int64_t batch, double beta, uint64_t seed, int64_t counter,
                               bool local) {
    c10::cuda::CUDAGuard guard(device_);
    const auto f = at::TensorOptions().dtype(at::kFloat).device(at::kCUDA, device_);
    at::Tensor out = at::empty({batch, row_dim_}, f.dtype(row_dtype_));
    at::Tensor ic = at::empty({batch + 1}, f.dtype(at::kLong));  // idx, then the count
    at::Tensor w = at::empty({batch}, f);
    at::Tensor pos = at::empty({batch}, f.dtype(at::kInt));
    at::Tensor idx = ic.narrow(0, 0, batch), count = ic.narrow(0, batch, 1);
    const int rc = (local ? per_sample_sharded_p2p_local_rng : per_sample_sharded_p2p_rng)(
        store_, rank, world, shard_base, reinterpret_cast<void* const*>(mailboxes), seed,
        reinterpret_cast<uint64_t*>(counter), batch, static_cast<float>(beta),
        rows(out), row_dim_, idx.data_ptr<int64_t>(), w.data_ptr<float>(),
        pos.data_ptr<int32_t>(), count.data_ptr<int64_t>(), stream());
    return py::make_tuple(rc, views(out), idx, w, pos, count);
  }

  // sample_sharded_p2p into caller-owned device buffers -> rc (rows
  // row_stride elements apart, idx int64, w float32, pos int32, count int64[1])
  int sample_sharded_p2p_into(int32_t rank, int32_t world, int64_t shard_base, int64_t mailboxes,
                              int64_t batch, double beta, uint64_t seed, int64_t counter,
                              int64_t rows_ptr, int64_t row_stride, int64_t idx, int64_t w,
                              int64_t pos, int64_t count, bool local) {
    c10::cuda::CUDAGuard guard(device_);
    return (local ? per_sample_sharded_p2p_local_rng : per_sample_sharded_p2p_rng)(
        store_, rank, world, shard_base, reinterpret_cast<void* const*>(mailboxes), seed,
        reinterpret_cast<uint64_t*>(counter), batch, static_cast<float>(beta),
        reinterpret_cast<float*>(rows_ptr), row_stride, reinterpret_cast<int64_t*>(idx),
        reinterpret_cast<float*>(w), reinterpret_cast<int32_t*>(pos),
        reinterpret_cast<int64_t*>(count), stream());
  }

  // sharded update of the first *count entries (global indices) -> rc
  int update_shard_count(int64_t base, const at::Tensor& idx, const at::Tensor& td,
                         const at::Tensor& count) {
    c10::cuda::CUDAGuard guard(device_);
    return per_update_priorities_shard_count(store_, base, idx.data_ptr<int64_t>(),
                                             td.data_ptr<float>(), idx.numel(),
                                             count.data_ptr<int64_t>(), stream());
  }

  // update_priorities(indices, td_errors) as the caller passes them: when both
  // are already what the C ABI takes (int64 / float32, contiguous, on this
  // device, as many TD errors as indices) -> rc of the update; otherwise -1
  // (nothing launched: the Python side converts them first). All checks are
  // C++ attribute reads, no tensor is made.
  int update_any(const at::Tensor& idx, const at::Tensor& td) {
    if (!idx.is_cuda() || !td.is_cuda() || idx.get_device() != device_ ||
        td.get_device() != device_ || idx.scalar_type() != at::kLong ||
        td.scalar_type() != at::kFloat || !idx.is_contiguous() || !td.is_contiguous() ||
        idx.numel() != td.numel() || idx.numel() == 0)
      return -1;
    c10::cuda::CUDAGuard guard(device_);
    return per_update_priorities(store_, idx.data_ptr<int64_t>(), td.data_ptr<float>(),
                                 idx.numel(), stream());
  }

  // update(idx int64, td float32), both contiguous on the device -> rc
  int update(const at::Tensor& idx, const at::Tensor& td) {
    c10::cuda::CUDAGuard guard(device_);
    return per_update_priorities(store_, idx.data_ptr<int64_t>(), td.data_ptr<float>(),
                                 idx.numel(), stream());
  }

 private:
  void* stream() const { return c10::cuda::getCurrentCUDAStream(device_).stream(); }

  // the output rows as the C ABI's pointer (float32 or 16-bit elements)
  static float* rows(const at::Tensor& out) { return static_cast<float*>(out.data_ptr()); }

  void alloc(int64_t batch, at::Tensor* out, at::Tensor* idx, at::Tensor* w) const {
    const auto f = at::TensorOptions().dtype(at::kFloat).device(at::kCUDA, device_);
    *out = at::empty({batch, row_dim_}, f.dtype(row_dtype_));
    *idx = at::empty({batch}, f.dtype(at::kLong));
    *w = at::empty({batch}, f);
  }

  py::dict views(const at::Tensor& out) const {
    py::dict d;
    const auto parts = out.split_with_sizes(dims_, 1);
    for (size_t k = 0; k < parts.size(); ++k) d[py_names_[k]] = parts[k];
    return d;
  }

  const per_store_t* store_;
  at::ScalarType row_dtype_;
  c10::DeviceIndex device_;
  std::vector<std::string> names_;
  std::vector<int64_t> dims_;
  py::list py_names_;
  uint64_t* counter_;
  int64_t row_dim_;
};

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "torch-tensor binding of the per_b200 sample / update calls";
  py::class_<Engine>(m, "Engine")
      .def(py::init<int64_t, int64_t, std::vector<std::string>, std::vector<int64_t>, int64_t,
                    int64_t>())
      .def("sample", &Engine::sample)
      .def("sample_into", &Engine::sample_into)
      .def("sample_from", &Engine::sample_from)
      .def("update", &Engine::update)
      .def("update_any", &Engine::update_any)
      .def("sample_sharded_p2p", &Engine::sample_sharded_p2p)
      .def("sample_sharded_p2p_into", &Engine::sample_sharded_p2p_into)
      .def("update_shard_count", &Engine::update_shard_count);
}
