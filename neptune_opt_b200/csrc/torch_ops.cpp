// The region ops registered with the PyTorch dispatcher from C++ (namespace `nb200`), so that a
// graph holding them can be compiled by AOTInductor into a package whose calls reach the CUDA
// kernels without any Python: the package's generated code calls the op by name through the
// dispatcher, and this library -- loaded into the process that runs the package -- answers with a
// C++ kernel that calls the C ABI of libneptune_b200.so (include/neptune_b200.h).
//
// Ops (CUDA kernels + Meta kernels that compute shapes only, for export and fake tensors):
//   fold(Tensor x, int skeleton, float[] params, bool keepdim, int plan, int block,
//        int num_warps=0) -> Tensor
//       params = [tiny, alpha, T, beta, N, eps]; plan 0 serial, 1 split (block-column chunks);
//       serial launch from num_warps as the host launch policy maps (block, num_warps): 0 the
//       library's own choice, 1 one warp per row, 2..16 one CTA of 32 n threads per row, 32 one
//       thread-block cluster per row
//   softmax(Tensor x, int mode) -> (Tensor y, Tensor lse)           mode 0 softmax, 1 log_softmax
//   l2_normalize(Tensor x) -> (Tensor y, Tensor norm)
//   rms_norm(Tensor x, Tensor gamma, float eps) -> Tensor
//   segment_pool(Tensor data, Tensor segments, bool offsets, int reduce, float? initial,
//                bool unsafe) -> Tensor                              reduce 0 sum, 1 mean
//   segment_status(int device, bool clear) -> int
//   segment_status_word(int device) -> Tensor      the per-device int32 word itself, for launches
//                                                  made through the C ABI by other host code
//   attention(Tensor q, Tensor k, Tensor v, bool causal, float scale) -> (Tensor o, Tensor lse)
//
// libneptune_b200.so is opened at the first call from the directory this library lives in, so
// the two files only need to sit side by side.
#include <dlfcn.h>

#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/csrc/inductor/aoti_torch/utils.h>
#include <torch/library.h>

#include <cstring>
#include <map>
#include <mutex>
#include <string>

#include "../../include/neptune_b200.h"

namespace {

struct Api {
    decltype(&nb200_last_error) last_error;
    decltype(&nb200_fold) fold;
    decltype(&nb200_fold_split_scratch_bytes) split_scratch_bytes;
    decltype(&nb200_fold_split) fold_split;
    decltype(&nb200_softmax) softmax;
    decltype(&nb200_l2_normalize) l2_normalize;
    decltype(&nb200_rms_norm) rms_norm;
    decltype(&nb200_segment_spans) segment_spans;
    decltype(&nb200_segment_pool) segment_pool;
    decltype(&nb200_attention) attention;
};

std::string own_directory() {
    Dl_info info;
    if (dladdr(reinterpret_cast<void*>(&own_directory), &info) && info.dli_fname) {
        std::string p(info.dli_fname);
        const auto slash = p.rfind('/');
        if (slash != std::string::npos) return p.substr(0, slash);
    }
    return ".";
}

template <typename F>
void bind(void* h, const char* name, F& f) {
    f = reinterpret_cast<F>(dlsym(h, name));
    TORCH_CHECK(f != nullptr, "nb200: libneptune_b200.so does not export ", name);
}

const Api& api() {
    static Api a;
    static std::once_flag once;
    std::call_once(once, [] {
        const std::string path = own_directory() + "/libneptune_b200.so";
        void* h = dlopen(path.c_str(), RTLD_NOW | RTLD_GLOBAL);
        TORCH_CHECK(h != nullptr, "nb200: cannot load ", path, ": ", dlerror());
        bind(h, "nb200_last_error", a.last_error);
        bind(h, "nb200_fold", a.fold);
        bind(h, "nb200_fold_split_scratch_bytes", a.split_scratch_bytes);
        bind(h, "nb200_fold_split", a.fold_split);
        bind(h, "nb200_softmax", a.softmax);
        bind(h, "nb200_l2_normalize", a.l2_normalize);
        bind(h, "nb200_rms_norm", a.rms_norm);
        bind(h, "nb200_segment_spans", a.segment_spans);
        bind(h, "nb200_segment_pool", a.segment_pool);
        bind(h, "nb200_attention", a.attention);
    });
    return a;
}

// Status codes to the exception types the Python layer raises for the same conditions.
void check(int rc, const char* what) {
    if (rc == NB200_OK) return;
    const char* msg = api().last_error();
    TORCH_CHECK_VALUE(rc != NB200_ERR_ARG, what, ": ", msg);
    TORCH_CHECK_NOT_IMPLEMENTED(rc != NB200_ERR_CAPACITY && rc != NB200_ERR_UNSUPPORTED, what, ": ", msg);
    TORCH_CHECK(false, what, ": ", msg);
}

int dtype_code(const at::Tensor& t) {
    switch (t.scalar_type()) {
        case at::kFloat: return NB200_F32;
        case at::kBFloat16: return NB200_BF16;
        case at::kHalf: return NB200_F16;
        default: TORCH_CHECK_TYPE(false, "nb200: dtype must be float32, bfloat16 or float16, got ", t.scalar_type());
    }
    return -1;
}

void* stream_of(const at::Tensor& t) { return c10::cuda::getCurrentCUDAStream(t.device().index()).stream(); }

// Rows of the last dimension: [..., n] viewed as [rows, n] (a copy only when no view exists).
at::Tensor rows_view(const at::Tensor& x) {
    TORCH_CHECK_VALUE(x.dim() >= 1, "nb200: input needs at least one dimension");
    TORCH_CHECK(x.size(-1) > 0, "nb200: the reduced width must be positive");
    return x.reshape({-1, x.size(-1)});
}

std::vector<int64_t> lead_shape(const at::Tensor& x, bool keepdim) {
    std::vector<int64_t> s(x.sizes().begin(), x.sizes().end() - 1);
    if (keepdim) s.push_back(1);
    return s;
}

nb200_params params_of(at::ArrayRef<double> p) {
    TORCH_CHECK_VALUE(p.size() == 6, "nb200.fold: params must be [tiny, alpha, T, beta, N, eps]");
    return nb200_params{p[0], p[1], p[2], p[3], p[4], p[5]};
}

void check_cuda(const at::Tensor& t, const char* what) {
    TORCH_CHECK_VALUE(t.is_cuda(), what, ": inputs must be CUDA tensors, got ", t.device());
}

// ------------------------------------------------------------------ CUDA kernels
// The launch a (block, num_warps) pair selects for the serial plan (nullptr: library default).
const nb200_launch* serial_launch(int64_t num_warps, nb200_launch* storage) {
    if (num_warps <= 0) return nullptr;
    if (num_warps == 1) {
        *storage = nb200_launch{NB200_VARIANT_WARP_ROW, 0, 0, 0};
    } else if (num_warps == 32) {
        *storage = nb200_launch{NB200_VARIANT_CLUSTER, 0, 0, 0};
    } else {
        TORCH_CHECK_VALUE(num_warps <= 16, "nb200.fold: num_warps must be in 0..16 or 32, got ", num_warps);
        *storage = nb200_launch{NB200_VARIANT_CTA_ROW, (int32_t)(32 * num_warps), 0, 0};
    }
    return storage;
}

at::Tensor fold_cuda(const at::Tensor& x, int64_t skeleton, at::ArrayRef<double> params, bool keepdim, int64_t plan,
                     int64_t block, int64_t num_warps) {
    check_cuda(x, "nb200.fold");
    const int dt = dtype_code(x);
    c10::cuda::CUDAGuard guard(x.device());
    const nb200_params p = params_of(params);
    at::Tensor out = at::empty(lead_shape(x, keepdim), x.options());
    if (out.numel() == 0) return out;
    const at::Tensor x2 = rows_view(x);
    if (plan == 0) {
        nb200_launch storage;
        check(api().fold((int)skeleton, &p, x2.data_ptr(), dt, x2.size(0), x2.size(1), x2.stride(0), x2.stride(1),
                         out.data_ptr(), serial_launch(num_warps, &storage), stream_of(x)),
              "nb200.fold");
    } else {
        const int64_t chunk = block > 0 ? block : 16384;
        const int64_t nparts = (x2.size(1) + chunk - 1) / chunk;
        const int64_t bytes = api().split_scratch_bytes(x2.size(0), nparts);
        TORCH_CHECK_NOT_IMPLEMENTED(bytes >= 0, "nb200.fold: split plan capacity: ", api().last_error());
        at::Tensor scratch = at::empty({std::max<int64_t>(bytes, 1)}, x.options().dtype(at::kByte));
        check(api().fold_split((int)skeleton, &p, x2.data_ptr(), dt, x2.size(0), x2.size(1), x2.stride(0),
                               x2.stride(1), chunk, scratch.data_ptr(), bytes, out.data_ptr(), nullptr, stream_of(x)),
              "nb200.fold");
    }
    return out;
}

std::tuple<at::Tensor, at::Tensor> softmax_cuda(const at::Tensor& x, int64_t mode) {
    check_cuda(x, "nb200.softmax");
    const int dt = dtype_code(x);
    c10::cuda::CUDAGuard guard(x.device());
    at::Tensor y = at::empty(x.sizes(), x.options());
    at::Tensor lse = at::empty(lead_shape(x, false), x.options());
    if (x.numel() == 0) return {y, lse};
    const at::Tensor x2 = rows_view(x);
    check(api().softmax((int)mode, x2.data_ptr(), dt, x2.size(0), x2.size(1), x2.stride(0), x2.stride(1),
                        y.data_ptr(), lse.data_ptr(), nullptr, stream_of(x)),
          "nb200.softmax");
    return {y, lse};
}

std::tuple<at::Tensor, at::Tensor> l2_cuda(const at::Tensor& x) {
    check_cuda(x, "nb200.l2_normalize");
    const int dt = dtype_code(x);
    c10::cuda::CUDAGuard guard(x.device());
    at::Tensor y = at::empty(x.sizes(), x.options());
    at::Tensor norm = at::empty(lead_shape(x, false), x.options());
    if (x.numel() == 0) return {y, norm};
    const at::Tensor x2 = rows_view(x);
    check(api().l2_normalize(x2.data_ptr(), dt, x2.size(0), x2.size(1), x2.stride(0), x2.stride(1), y.data_ptr(),
                             norm.data_ptr(), nullptr, stream_of(x)),
          "nb200.l2_normalize");
    return {y, norm};
}

at::Tensor rms_cuda(const at::Tensor& x, const at::Tensor& gamma, double eps) {
    check_cuda(x, "nb200.rms_norm");
    check_cuda(gamma, "nb200.rms_norm");
    const int dt = dtype_code(x);
    TORCH_CHECK_TYPE(gamma.scalar_type() == x.scalar_type(), "nb200.rms_norm: gamma must have x's dtype");
    TORCH_CHECK_VALUE(gamma.dim() == 1 && x.dim() >= 1 && gamma.size(0) == x.size(-1),
                      "nb200.rms_norm: gamma must be 1-D with x's last dimension");
    c10::cuda::CUDAGuard guard(x.device());
    at::Tensor y = at::empty(x.sizes(), x.options());
    if (x.numel() == 0) return y;
    const at::Tensor x2 = rows_view(x);
    check(api().rms_norm(x2.data_ptr(), gamma.data_ptr(), dt, x2.size(0), x2.size(1), x2.stride(0), x2.stride(1),
                         gamma.stride(0), eps, y.data_ptr(), nullptr, stream_of(x)),
          "nb200.rms_norm");
    return y;
}

// Per-device descriptor-status words of the C++ ops (same bits as the Python layer's:
// 1 negative or oversized length, 2 lengths not covering the rows, 4 boundary out of range,
// 8 boundaries decreasing). Malformed segments pool to NaN; the word records why.
std::mutex g_status_mutex;
std::map<int, at::Tensor> g_status;

at::Tensor status_word(const at::Device& dev) {
    std::lock_guard<std::mutex> lock(g_status_mutex);
    auto it = g_status.find(dev.index());
    if (it != g_status.end()) return it->second;
    at::Tensor w = at::zeros({1}, at::TensorOptions().dtype(at::kInt).device(dev));
    g_status.emplace(dev.index(), w);
    return w;
}

int index_code(const at::Tensor& t) {
    if (t.scalar_type() == at::kInt) return NB200_I32;
    TORCH_CHECK_TYPE(t.scalar_type() == at::kLong, "nb200.segment_pool: segments must be int32 or int64");
    return NB200_I64;
}

at::Tensor segment_cuda(const at::Tensor& data, const at::Tensor& segments, bool offsets, int64_t reduce,
                        std::optional<double> initial, bool unsafe) {
    check_cuda(data, "nb200.segment_pool");
    check_cuda(segments, "nb200.segment_pool");
    const int dt = dtype_code(data);
    const int idt = index_code(segments);
    TORCH_CHECK_VALUE(data.dim() >= 1 && segments.dim() == 1, "nb200.segment_pool: data [T, ...], segments 1-D");
    TORCH_CHECK_VALUE(reduce == 0 || reduce == 1, "nb200.segment_pool: reduce must be 0 (sum) or 1 (mean)");
    TORCH_CHECK_VALUE(!offsets || segments.size(0) >= 1, "nb200.segment_pool: offsets need at least one boundary");
    c10::cuda::CUDAGuard guard(data.device());
    const int64_t nseg = offsets ? segments.size(0) - 1 : segments.size(0);
    std::vector<int64_t> shape{nseg};
    int64_t channels = 1;
    for (int64_t d = 1; d < data.dim(); ++d) {
        shape.push_back(data.size(d));
        channels *= data.size(d);
    }
    at::Tensor out = at::empty(shape, data.options());
    if (nseg == 0 || channels == 0) return out;
    at::Tensor status = status_word(data.device());
    void* st = stream_of(data);
    at::Tensor bounds = segments;
    int bidx = idt;
    int64_t bstride = segments.numel() ? segments.stride(0) : 1;
    if (!offsets) {
        bounds = at::empty({nseg + 1}, segments.options().dtype(at::kLong));
        check(api().segment_spans(segments.data_ptr(), idt, nseg, bstride, unsafe ? 1 : 0, data.size(0),
                                  bounds.data_ptr<int64_t>(), reinterpret_cast<uint32_t*>(status.data_ptr()), st),
              "nb200.segment_pool");
        bidx = NB200_I64;
        bstride = 1;
    }
    const at::Tensor flat = data.reshape({data.size(0), channels});
    uint32_t bits = 0;
    if (initial.has_value()) {
        const float f = static_cast<float>(*initial);
        std::memcpy(&bits, &f, sizeof(bits));
    }
    check(api().segment_pool(flat.data_ptr(), dt, flat.size(0), channels, flat.stride(0), flat.stride(1),
                             bounds.data_ptr(), bidx, bstride, nseg, (int)reduce, initial.has_value() ? 1 : 0, bits,
                             out.data_ptr(), reinterpret_cast<uint32_t*>(status.data_ptr()), st),
          "nb200.segment_pool");
    return out;
}

at::Tensor segment_status_word(int64_t device) { return status_word(at::Device(at::kCUDA, (c10::DeviceIndex)device)); }

int64_t segment_status(int64_t device, bool clear) {
    at::Tensor w = status_word(at::Device(at::kCUDA, (c10::DeviceIndex)device));
    const int64_t bits = w.item<int32_t>();
    if (clear && bits) w.zero_();
    return bits;
}

std::tuple<at::Tensor, at::Tensor> attention_cuda(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                                  bool causal, double scale) {
    check_cuda(q, "nb200.attention");
    TORCH_CHECK_TYPE(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 &&
                         v.scalar_type() == at::kBFloat16,
                     "nb200.attention: q, k, v must be bfloat16");
    TORCH_CHECK_VALUE(q.dim() == 4 && q.sizes() == k.sizes() && q.sizes() == v.sizes(),
                      "nb200.attention: q, k, v must share one [batch, heads, seq, head_dim] shape");
    c10::cuda::CUDAGuard guard(q.device());
    const at::Tensor qc = q.contiguous(), kc = k.contiguous(), vc = v.contiguous();
    at::Tensor o = at::empty(q.sizes(), q.options());
    at::Tensor lse = at::empty({q.size(0), q.size(1), q.size(2)}, q.options().dtype(at::kFloat));
    if (q.numel() == 0) return {o, lse};
    check(api().attention(qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), o.data_ptr(), lse.data_ptr<float>(), q.size(0),
                          q.size(1), q.size(2), q.size(3), causal ? 1 : 0, (float)scale, stream_of(q)),
          "nb200.attention");
    return {o, lse};
}

// ------------------------------------------------------------------ Meta kernels (shapes only)
// Symbolic sizes throughout, so graphs exported with dynamic dimensions trace through these ops.
std::vector<c10::SymInt> lead_sym_shape(const at::Tensor& x, bool keepdim) {
    const auto s = x.sym_sizes();
    std::vector<c10::SymInt> v(s.begin(), s.end() - 1);
    if (keepdim) v.emplace_back(1);
    return v;
}
at::Tensor fold_meta(const at::Tensor& x, int64_t, at::ArrayRef<double>, bool keepdim, int64_t, int64_t, int64_t) {
    return at::empty_symint(lead_sym_shape(x, keepdim), x.options());
}
std::tuple<at::Tensor, at::Tensor> softmax_meta(const at::Tensor& x, int64_t) {
    return {at::empty_symint(x.sym_sizes(), x.options()), at::empty_symint(lead_sym_shape(x, false), x.options())};
}
std::tuple<at::Tensor, at::Tensor> l2_meta(const at::Tensor& x) {
    return {at::empty_symint(x.sym_sizes(), x.options()), at::empty_symint(lead_sym_shape(x, false), x.options())};
}
at::Tensor rms_meta(const at::Tensor& x, const at::Tensor&, double) {
    return at::empty_symint(x.sym_sizes(), x.options());
}
at::Tensor segment_meta(const at::Tensor& data, const at::Tensor& segments, bool offsets, int64_t,
                        std::optional<double>, bool) {
    std::vector<c10::SymInt> shape{offsets ? segments.sym_size(0) - 1 : segments.sym_size(0)};
    const auto ds = data.sym_sizes();
    for (size_t d = 1; d < ds.size(); ++d) shape.push_back(ds[d]);
    return at::empty_symint(shape, data.options());
}
std::tuple<at::Tensor, at::Tensor> attention_meta(const at::Tensor& q, const at::Tensor&, const at::Tensor&, bool,
                                                  double) {
    const auto qs = q.sym_sizes();
    return {at::empty_symint(qs, q.options()),
            at::empty_symint(std::vector<c10::SymInt>(qs.begin(), qs.end() - 1), q.options().dtype(at::kFloat))};
}

}  // namespace

// ------------------------------------------------------------------ AOTInductor C shims
// Direct C entry points for AOTInductor packages (torch._inductor.config.aot_inductor.
// custom_ops_to_c_shims): a package compiled with them calls these functions instead of going
// through the proxy executor's boxed dispatcher call, which costs microseconds per region call.
// Argument conventions are AOTInductor's generated C shims': tensors as AtenTensorHandle, int as
// int64_t, bool as int32_t, float as double, float? as double* (nullptr = None), float[] as pointer
// + length, results as AtenTensorHandle* out-parameters. The process that runs such a package
// must make these symbols visible (load this library with RTLD_GLOBAL, as aot.load() does).
namespace {
at::Tensor& tensor_of(AtenTensorHandle h) { return *torch::aot_inductor::tensor_handle_to_tensor_pointer(h); }
}  // namespace

extern "C" {
AOTITorchError aoti_torch_cuda_fold(AtenTensorHandle x, int64_t skeleton, const double* params, int64_t params_len_,
                                    int32_t keepdim, int64_t plan, int64_t block, int64_t num_warps,
                                    AtenTensorHandle* ret0) {
    AOTI_TORCH_CONVERT_EXCEPTION_TO_ERROR_CODE({
        *ret0 = torch::aot_inductor::new_tensor_handle(fold_cuda(tensor_of(x), skeleton,
                                                                 at::ArrayRef<double>(params, params_len_),
                                                                 keepdim != 0, plan, block, num_warps));
    });
}
AOTITorchError aoti_torch_cuda_softmax(AtenTensorHandle x, int64_t mode, AtenTensorHandle* ret0,
                                       AtenTensorHandle* ret1) {
    AOTI_TORCH_CONVERT_EXCEPTION_TO_ERROR_CODE({
        auto r = softmax_cuda(tensor_of(x), mode);
        *ret0 = torch::aot_inductor::new_tensor_handle(std::move(std::get<0>(r)));
        *ret1 = torch::aot_inductor::new_tensor_handle(std::move(std::get<1>(r)));
    });
}
AOTITorchError aoti_torch_cuda_l2_normalize(AtenTensorHandle x, AtenTensorHandle* ret0, AtenTensorHandle* ret1) {
    AOTI_TORCH_CONVERT_EXCEPTION_TO_ERROR_CODE({
        auto r = l2_cuda(tensor_of(x));
        *ret0 = torch::aot_inductor::new_tensor_handle(std::move(std::get<0>(r)));
        *ret1 = torch::aot_inductor::new_tensor_handle(std::move(std::get<1>(r)));
    });
}
AOTITorchError aoti_torch_cuda_rms_norm(AtenTensorHandle x, AtenTensorHandle gamma, double eps,
                                        AtenTensorHandle* ret0) {
    AOTI_TORCH_CONVERT_EXCEPTION_TO_ERROR_CODE({
        *ret0 = torch::aot_inductor::new_tensor_handle(rms_cuda(tensor_of(x), tensor_of(gamma), eps));
    });
}
AOTITorchError aoti_torch_cuda_segment_pool(AtenTensorHandle data, AtenTensorHandle segments, int32_t offsets,
                                            int64_t reduce, double* initial, int32_t unsafe, AtenTensorHandle* ret0) {
    AOTI_TORCH_CONVERT_EXCEPTION_TO_ERROR_CODE({
        const std::optional<double> init = initial ? std::optional<double>(*initial) : std::nullopt;
        *ret0 = torch::aot_inductor::new_tensor_handle(
            segment_cuda(tensor_of(data), tensor_of(segments), offsets != 0, reduce, init, unsafe != 0));
    });
}
AOTITorchError aoti_torch_cuda_attention(AtenTensorHandle q, AtenTensorHandle k, AtenTensorHandle v, int32_t causal,
                                         double scale, AtenTensorHandle* ret0, AtenTensorHandle* ret1) {
    AOTI_TORCH_CONVERT_EXCEPTION_TO_ERROR_CODE({
        auto r = attention_cuda(tensor_of(q), tensor_of(k), tensor_of(v), causal != 0, scale);
        *ret0 = torch::aot_inductor::new_tensor_handle(std::move(std::get<0>(r)));
        *ret1 = torch::aot_inductor::new_tensor_handle(std::move(std::get<1>(r)));
    });
}
}  // extern "C"

TORCH_LIBRARY(nb200, m) {
    m.def("fold(Tensor x, int skeleton, float[] params, bool keepdim, int plan, int block, int num_warps=0) -> Tensor");
    m.def("softmax(Tensor x, int mode) -> (Tensor, Tensor)");
    m.def("l2_normalize(Tensor x) -> (Tensor, Tensor)");
    m.def("rms_norm(Tensor x, Tensor gamma, float eps) -> Tensor");
    m.def("segment_pool(Tensor data, Tensor segments, bool offsets, int reduce, float? initial, bool unsafe) -> Tensor");
    m.def("segment_status(int device, bool clear) -> int", &segment_status);
    m.def("segment_status_word(int device) -> Tensor", &segment_status_word);
    m.def("attention(Tensor q, Tensor k, Tensor v, bool causal, float scale) -> (Tensor, Tensor)");
}

TORCH_LIBRARY_IMPL(nb200, CUDA, m) {
    m.impl("fold", &fold_cuda);
    m.impl("softmax", &softmax_cuda);
    m.impl("l2_normalize", &l2_cuda);
    m.impl("rms_norm", &rms_cuda);
    m.impl("segment_pool", &segment_cuda);
    m.impl("attention", &attention_cuda);
}

TORCH_LIBRARY_IMPL(nb200, Meta, m) {
    m.impl("fold", &fold_meta);
    m.impl("softmax", &softmax_meta);
    m.impl("l2_normalize", &l2_meta);
    m.impl("rms_norm", &rms_meta);
    m.impl("segment_pool", &segment_meta);
    m.impl("attention", &attention_meta);
}
