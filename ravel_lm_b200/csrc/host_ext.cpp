// Python binding of the host calls that run once per decode step or per lookup.
//
// A decode step (RavelLayerCache.step) launches one short kernel; through
// ctypes its Python side -- fourteen argument conversions, the dtype / device /
// layout checks and two output allocations -- took longer than the kernel.
// Here the checks, the allocations (the caching allocator through ATen) and the
// C-ABI call run in C++: the Python caller makes one call.  The lookup entry
// points (tape build, latest-k and segmented-sum forward and backward) get the
// same treatment.
//
// Every function here does exactly what the ctypes path in ravel_memory.py does
// with the same arguments: same entry point of libravel_b200.so, same sizes,
// same stream (the current stream of the tensors' device).  Failure statuses are
// returned to the caller, which raises the library's own errors.  The cache step
// returns None when its arguments are not the common case (the caller then
// takes the fully checked Python path, with its error messages).

#include <ATen/ATen.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/csrc/autograd/python_variable.h>
#include <torch/csrc/utils/pybind.h>

#include <optional>
#include <tuple>

#include "../../include/ravel_b200.h"

namespace py = pybind11;

namespace {

int payload_code(at::ScalarType t) {
    switch (t) {
        case at::kFloat: return RAVEL_F32;
        case at::kBFloat16: return RAVEL_BF16;
        case at::kHalf: return RAVEL_F16;
        case at::kDouble: return RAVEL_F64;
        default: return -1;
    }
}

void* stream_of(const at::Tensor& t) { return c10::cuda::getCurrentCUDAStream(t.device().index()).stream(); }

const void* ptr_or_null(const std::optional<at::Tensor>& t) { return t ? t->data_ptr() : nullptr; }

at::Tensor bytes(size_t n, const at::Tensor& like) {
    return at::empty({static_cast<int64_t>(n)}, like.options().dtype(at::kByte));
}

// RavelLayerCache.step for contiguous CUDA tensors on one device, addresses
// int64 or int32 of one type, payloads in the cache dtype, out None or a
// matching (values, mask) pair.  Returns (values, mask), an int status on a
// library failure, or None for any other argument combination.
py::object cache_step(const at::Tensor& values, const at::Tensor& filled, const at::Tensor& ra, const at::Tensor& wa,
                      const at::Tensor& payloads, const py::object& out) {
    if (!values.is_cuda() || values.dim() != 4 || filled.dim() != 3 || ra.dim() != 2 || wa.dim() != 2 ||
        payloads.dim() != 3)
        return py::none();
    const auto dev = values.device();
    if (filled.device() != dev || ra.device() != dev || wa.device() != dev || payloads.device() != dev)
        return py::none();
    const auto adt = ra.scalar_type();
    if ((adt != at::kLong && adt != at::kInt) || wa.scalar_type() != adt) return py::none();
    const int code = payload_code(values.scalar_type());
    if (code < 0 || payloads.scalar_type() != values.scalar_type() || filled.scalar_type() != at::kBool)
        return py::none();
    if (!values.is_contiguous() || !filled.is_contiguous() || !ra.is_contiguous() || !wa.is_contiguous() ||
        !payloads.is_contiguous())
        return py::none();
    const int64_t B = ra.size(0), C = ra.size(1), A = values.size(2), D = values.size(3);
    if (wa.size(0) != B || wa.size(1) != C || values.size(0) != B || values.size(1) != C || payloads.size(0) != B ||
        payloads.size(1) != C || payloads.size(2) != D || filled.size(0) != B || filled.size(1) != C ||
        filled.size(2) != A)
        return py::none();
    at::Tensor vals, mask;
    if (out.is_none()) {
        vals = at::empty({B, C, D}, values.options());
        mask = at::empty({B, C}, filled.options());
    } else {
        if (!py::isinstance<py::tuple>(out) && !py::isinstance<py::list>(out)) return py::none();
        const py::sequence seq = out.cast<py::sequence>();
        if (seq.size() != 2 || !THPVariable_Check(seq[0].ptr()) || !THPVariable_Check(seq[1].ptr()))
            return py::none();
        vals = THPVariable_Unpack(seq[0].ptr());
        mask = THPVariable_Unpack(seq[1].ptr());
        if (vals.dim() != 3 || vals.size(0) != B || vals.size(1) != C || vals.size(2) != D ||
            vals.scalar_type() != values.scalar_type() || vals.device() != dev || !vals.is_contiguous() ||
            mask.dim() != 2 || mask.size(0) != B || mask.size(1) != C || mask.scalar_type() != at::kBool ||
            mask.device() != dev || !mask.is_contiguous())
            return py::none();
    }
    const int rc = ravel_cache_step(values.data_ptr(), static_cast<uint8_t*>(filled.data_ptr()), ra.data_ptr(),
                                    wa.data_ptr(), adt == at::kLong ? RAVEL_I64 : RAVEL_I32, payloads.data_ptr(),
                                    code, B, C, A, D, vals.data_ptr(), static_cast<uint8_t*>(mask.data_ptr()),
                                    stream_of(values));
    if (rc != RAVEL_OK) return py::int_(rc);
    return py::make_tuple(vals, mask);
}

// ravel_tape_build into a new tape and a scratch buffer sized for a lookup of
// payload width D, dtype code dcode and k.  Returns (status, tape, scratch).
std::tuple<int, at::Tensor, at::Tensor> tape_build(const at::Tensor& w, const std::optional<at::Tensor>& r, int code,
                                                   const std::optional<at::Tensor>& mask, int64_t A, int flags,
                                                   int64_t D, int64_t k, int dcode) {
    const int64_t B = w.size(0), T = w.size(1), C = w.size(2);
    const size_t tb = ravel_tape_bytes(B, T, C, A, flags), sb = ravel_scratch_bytes(B, T, C, D, A, k, dcode, flags);
    at::Tensor tape = bytes(tb, w), scratch = bytes(sb, w);
    const int rc = ravel_tape_build(w.data_ptr(), ptr_or_null(r), code,
                                    static_cast<const uint8_t*>(ptr_or_null(mask)), B, T, C, A, flags,
                                    tape.data_ptr(), tb, scratch.data_ptr(), sb, stream_of(w));
    return {rc, tape, scratch};
}

// ravel_latestk_fwd_tape into new [B,T,C,k,D] values and [B,T,C,k] mask.
std::tuple<int, at::Tensor, at::Tensor> latestk_fwd(const at::Tensor& tape, int flags,
                                                    const std::optional<at::Tensor>& r, int code,
                                                    const at::Tensor& p, int64_t B, int64_t T, int64_t C, int64_t A,
                                                    int64_t k) {
    const int64_t D = p.size(-1);
    at::Tensor vals = at::empty({B, T, C, k, D}, p.options());
    at::Tensor mask = at::empty({B, T, C, k}, p.options().dtype(at::kBool));
    const int rc = ravel_latestk_fwd_tape(tape.data_ptr(), flags, ptr_or_null(r), code, p.data_ptr(),
                                          payload_code(p.scalar_type()), B, T, C, D, A, k, vals.data_ptr(),
                                          static_cast<uint8_t*>(mask.data_ptr()), stream_of(p));
    return {rc, vals, mask};
}

// ravel_segsum_fwd_tape into new [B,T,C,D] sums and [B,T,C] mask.
std::tuple<int, at::Tensor, at::Tensor> segsum_fwd(const at::Tensor& tape, int flags,
                                                   const std::optional<at::Tensor>& r, int code, const at::Tensor& p,
                                                   const at::Tensor& scratch, int64_t B, int64_t T, int64_t C,
                                                   int64_t A) {
    const int64_t D = p.size(-1);
    at::Tensor sums = at::empty({B, T, C, D}, p.options());
    at::Tensor mask = at::empty({B, T, C}, p.options().dtype(at::kBool));
    const int rc = ravel_segsum_fwd_tape(tape.data_ptr(), flags, ptr_or_null(r), code, p.data_ptr(),
                                         payload_code(p.scalar_type()), B, T, C, D, A, sums.data_ptr(),
                                         static_cast<uint8_t*>(mask.data_ptr()), scratch.data_ptr(),
                                         static_cast<size_t>(scratch.numel()), stream_of(p));
    return {rc, sums, mask};
}

// ravel_segsum_bwd into a new [B,T,C,D] payload gradient.
std::tuple<int, at::Tensor> segsum_bwd(const at::Tensor& tape, int flags, const std::optional<at::Tensor>& r,
                                       int code, const at::Tensor& g, int64_t B, int64_t T, int64_t C, int64_t A) {
    const int64_t D = g.size(-1);
    const int dcode = payload_code(g.scalar_type());
    const size_t sb = ravel_scratch_bytes(B, T, C, D, A, 1, dcode, flags);
    at::Tensor grad = at::empty({B, T, C, D}, g.options());
    at::Tensor scratch = bytes(sb, g);
    const int rc = ravel_segsum_bwd(tape.data_ptr(), flags, ptr_or_null(r), code, g.data_ptr(), dcode, B, T, C, D, A,
                                    grad.data_ptr(), scratch.data_ptr(), sb, stream_of(g));
    return {rc, grad};
}

// ravel_latestk_bwd into a new payload gradient, or ravel_latestk_bwd_accumulate
// into acc (checked by the caller: contiguous [B,T,C,D] of the gradient dtype).
std::tuple<int, at::Tensor> latestk_bwd(const at::Tensor& tape, int flags, const std::optional<at::Tensor>& r,
                                        int code, const at::Tensor& g, int64_t B, int64_t T, int64_t C, int64_t A,
                                        int64_t k, const std::optional<at::Tensor>& acc) {
    const int64_t D = g.size(-1);
    const int dcode = payload_code(g.scalar_type());
    const size_t sb = ravel_scratch_bytes(B, T, C, D, A, k, dcode, flags);
    at::Tensor grad = acc ? *acc : at::empty({B, T, C, D}, g.options());
    at::Tensor scratch = bytes(sb, g);
    const int rc = (acc ? ravel_latestk_bwd_accumulate : ravel_latestk_bwd)(
        tape.data_ptr(), flags, ptr_or_null(r), code, g.data_ptr(), dcode, B, T, C, D, A, k, grad.data_ptr(),
        scratch.data_ptr(), sb, stream_of(g));
    return {rc, grad};
}

}  // namespace

PYBIND11_MODULE(_ravel_host, m) {
    m.doc() = "C++ host calls of libravel_b200 for the per-step Python paths";
    m.def("cache_step", &cache_step);
    m.def("tape_build", &tape_build);
    m.def("latestk_fwd", &latestk_fwd);
    m.def("segsum_fwd", &segsum_fwd);
    m.def("segsum_bwd", &segsum_bwd);
    m.def("latestk_bwd", &latestk_bwd);
}
