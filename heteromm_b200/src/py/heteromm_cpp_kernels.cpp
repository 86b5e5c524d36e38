// heteromm_cpp_kernels: Python bindings of the C++ step API, under the names
// the reference's pipeline generator emits for steps that have no Python
// implementation (toolchain/frontend/dev/passes/python_dispatch_pass.h:518-540,
// 695-712): `heteromm_cpp_kernels.<StepClass>_<kernel>(*args, **kwargs)`, with
// kernel "cpu" or "gpu", called as
//   build:     <Build>(retrieved_data, ...)                      -> memory
//   score:     <Score>(memory, query, ...)                        -> scores
//   retrieval: <Retrieval>(scores, ...)                           -> indices
//   apply:     <Apply>(query, retrieved_data, indices, input_data, ...) -> output
//   fused:     <Fused>(memory, query, ...)                        -> indices
// (python_dispatch_pass.h:732-830).  Step parameters (k, threshold, page_size,
// weight) come as keyword arguments; the generated pipeline passes one set of
// keyword arguments to every step, so each function ignores the ones it does
// not use.  Arrays are NumPy arrays (or anything NumPy converts).  The "gpu"
// functions run the GPU work of the step's KernelType::GPU arm (this library's
// CUDA kernels) and the "cpu" functions its CPU arm, with the Python lock
// released.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cmath>
#include <string>
#include <unordered_map>
#include <vector>

#include "heteromm/dev/steps/apply_memory.h"
#include "heteromm/dev/steps/build_memory.h"
#include "heteromm/dev/steps/compute_score.h"
#include "heteromm/dev/steps/fused_steps/template.h"
#include "heteromm/dev/steps/memory_retrieval.h"
#include "packed.h"

namespace py = pybind11;
using namespace heteromm;
using step::KernelType;

namespace {

using F32 = py::array_t<float, py::array::c_style | py::array::forcecast>;
using I32 = py::array_t<int, py::array::c_style | py::array::forcecast>;

std::vector<std::vector<float>> rows_of(const py::handle& obj, const char* what) {
    F32 a = F32::ensure(obj);
    if (!a || a.ndim() != 2) throw py::value_error(std::string(what) + " must be a 2-D float array");
    const size_t r = (size_t)a.shape(0), c = (size_t)a.shape(1);
    std::vector<std::vector<float>> m(r);
    const float* p = a.data();
    for (size_t i = 0; i < r; ++i) m[i].assign(p + i * c, p + (i + 1) * c);
    return m;
}

std::vector<float> vec_of(const py::handle& obj, const char* what) {
    F32 a = F32::ensure(obj);
    if (!a || a.ndim() != 1) throw py::value_error(std::string(what) + " must be a 1-D float array");
    return std::vector<float>(a.data(), a.data() + a.size());
}

std::vector<int> ints_of(const py::handle& obj, const char* what) {
    I32 a = I32::ensure(obj);
    if (!a || a.ndim() != 1) throw py::value_error(std::string(what) + " must be a 1-D integer array");
    return std::vector<int>(a.data(), a.data() + a.size());
}

py::array_t<float> to_array(const std::vector<float>& v) {
    py::array_t<float> a((py::ssize_t)v.size());
    std::copy(v.begin(), v.end(), a.mutable_data());
    return a;
}

py::array_t<int> to_array(const std::vector<int>& v) {
    py::array_t<int> a((py::ssize_t)v.size());
    std::copy(v.begin(), v.end(), a.mutable_data());
    return a;
}

py::array_t<float> to_array(const std::vector<std::vector<float>>& m) {
    const size_t r = m.size(), c = r ? m[0].size() : 0;
    py::array_t<float> a({(py::ssize_t)r, (py::ssize_t)c});
    float* p = a.mutable_data();
    for (size_t i = 0; i < r; ++i) std::copy(m[i].begin(), m[i].end(), p + i * c);
    return a;
}

// A keyword argument, or `fallback` when it is absent.
template <typename T>
T kw(const py::kwargs& kwargs, const char* name, T fallback) {
    return kwargs.contains(name) ? kwargs[name].cast<T>() : fallback;
}

template <typename T>
T kw_required(const py::kwargs& kwargs, const char* name, const char* fn) {
    if (!kwargs.contains(name))
        throw py::type_error(std::string(fn) + " needs the keyword argument '" + name + "'");
    return kwargs[name].cast<T>();
}

// KV cache data: a (keys, values) pair or a mapping with "keys" and "values".
data_type::KVCacheData<float> kv_of(const py::handle& obj) {
    data_type::KVCache<float> kv;
    if (py::isinstance<py::dict>(obj)) {
        py::dict d = py::reinterpret_borrow<py::dict>(obj);
        kv.keys = rows_of(d["keys"], "retrieved_data['keys']");
        kv.values = rows_of(d["values"], "retrieved_data['values']");
    } else {
        py::sequence s = py::reinterpret_borrow<py::sequence>(obj);
        if (py::len(s) != 2) throw py::value_error("retrieved_data must be (keys, values)");
        kv.keys = rows_of(s[0], "keys");
        kv.values = rows_of(s[1], "values");
    }
    return data_type::KVCacheData<float>(kv);
}

// BM25 index: a sequence of documents, each a {token id: term frequency}
// mapping (the reference's per-document maps, types/memory.h BM25IndexData).
data_type::BM25IndexMemory bm25_of(const py::handle& obj) {
    data_type::BM25IndexMemory mem;
    for (const py::handle& doc : py::reinterpret_borrow<py::sequence>(obj))
        mem.insert_document(doc.cast<std::unordered_map<int, int>>());
    return mem;
}

// BM25 query: a {token id: frequency} mapping, or a sequence of token ids.
data_type::BM25Query bm25_query_of(const py::handle& obj) {
    data_type::BM25QueryType q;
    if (py::isinstance<py::dict>(obj)) {
        q = obj.cast<data_type::BM25QueryType>();
    } else {
        for (const py::handle& t : py::reinterpret_borrow<py::sequence>(obj)) q[t.cast<int>()] += 1;
    }
    return data_type::BM25Query(q);
}

// `obj` as a C-contiguous 2-D float array with `cols` columns, if it is one.
bool matrix_with_cols(const py::handle& obj, size_t cols, F32& out) {
    F32 a = F32::ensure(obj);
    if (!a || a.ndim() != 2 || (size_t)a.shape(1) != cols) return false;
    out = a;
    return true;
}

// ------------------------------------------------------------------- steps
//
// The "gpu" functions hand NumPy's contiguous buffers straight to the GPU
// work of the step adapters (packed.h) when the shapes are the ones that work
// uses, which skips the vector-of-vectors copies of the step types; any other
// input goes through the step object, as the "cpu" functions always do.

py::array_t<float> inner_product(KernelType kt, const py::object& memory, const py::object& query,
                                 const py::kwargs&) {
    if (kt == KernelType::GPU) {
        const std::vector<float> q = vec_of(query, "query");
        F32 m;
        if (matrix_with_cols(memory, q.size(), m) && !q.empty()) {
            std::vector<float> out;
            {
                py::gil_scoped_release nogil;
                out = gpu::ip_scores(m.data(), (size_t)m.shape(0), q.size(), q.data());
            }
            return to_array(out);
        }
    }
    data_type::FlatIndexMemory<float> mem(rows_of(memory, "memory"));
    data_type::VectorQuery<float> q(vec_of(query, "query"));
    data_type::VectorScore<float> out;
    {
        py::gil_scoped_release nogil;
        step::InnerProductCompute s;
        s.set_current_kernel(kt);
        s.execute(mem, q, out);
    }
    return to_array(out.export_data());
}

py::array_t<int> topk(KernelType kt, const py::object& scores, const py::kwargs& kwargs) {
    data_type::VectorScore<float> sc(vec_of(scores, "scores"));
    const size_t k = kw<size_t>(kwargs, "k", 64);
    data_type::TopKIndex out;
    {
        py::gil_scoped_release nogil;
        step::TopKRetrieval s(k);
        s.set_current_kernel(kt);
        s.execute(sc, out);
    }
    return to_array(out.export_data());
}

py::array_t<int> threshold(KernelType kt, const py::object& scores, const py::kwargs& kwargs) {
    data_type::VectorScore<float> sc(vec_of(scores, "scores"));
    const float t = kw_required<float>(kwargs, "threshold", "ThresholdRetrieval");
    data_type::ThresholdBitmapIndex out;
    {
        py::gil_scoped_release nogil;
        step::ThresholdRetrieval s(t);
        s.set_current_kernel(kt);
        s.execute(sc, out);
    }
    return to_array(out.get_selected_indices());
}

py::array_t<int> ip_topk(KernelType kt, const py::object& memory, const py::object& query,
                         const py::kwargs& kwargs) {
    if (kt == KernelType::GPU) {
        const std::vector<float> q = vec_of(query, "query");
        F32 m;
        if (matrix_with_cols(memory, q.size(), m) && !q.empty()) {
            const size_t k = kw<size_t>(kwargs, "k", 64);
            std::vector<int> out;
            {
                py::gil_scoped_release nogil;
                out = gpu::ip_topk(m.data(), (size_t)m.shape(0), q.size(), q.data(), k);
            }
            return to_array(out);
        }
    }
    data_type::FlatIndexMemory<float> mem(rows_of(memory, "memory"));
    data_type::VectorQuery<float> q(vec_of(query, "query"));
    const size_t k = kw<size_t>(kwargs, "k", 64);
    data_type::TopKIndex out;
    {
        py::gil_scoped_release nogil;
        step::InnerProductTopKRetrieval s(k);
        s.set_kernel(kt);
        s.execute(mem, q, out);
    }
    return to_array(out.export_data());
}

// keys of (keys, values) or {"keys": ..., "values": ...}
py::object kv_part(const py::handle& obj, const char* name, size_t i) {
    if (py::isinstance<py::dict>(obj)) return py::reinterpret_borrow<py::dict>(obj)[name];
    return py::reinterpret_borrow<py::sequence>(obj)[i];
}

py::array_t<float> paged_builder(KernelType kt, const py::object& retrieved_data,
                                 const py::kwargs& kwargs) {
    if (kt == KernelType::GPU) {
        F32 keys = F32::ensure(kv_part(retrieved_data, "keys", 0));
        const int page = kw_required<int>(kwargs, "page_size", "PagedKVIndexBuilder");
        if (keys && keys.ndim() == 2 && keys.shape(0) > 0 && keys.shape(1) > 0 && page > 0) {
            const size_t L = (size_t)keys.shape(0), D = (size_t)keys.shape(1);
            F32 w;
            bool have_w = false;
            std::vector<float> eye;
            if (kwargs.contains("weight") && !kwargs["weight"].is_none()) {
                have_w = matrix_with_cols(kwargs["weight"], D, w);
            } else {
                eye.assign(D * D, 0.0f);
                for (size_t i = 0; i < D; ++i) eye[i * D + i] = 1.0f;
            }
            const size_t out_dim = have_w ? (size_t)w.shape(0) : (eye.empty() ? 0 : D);
            if (out_dim > 0) {
                const float* wp = have_w ? w.data() : eye.data();
                std::vector<float> flat;
                {
                    py::gil_scoped_release nogil;
                    flat = gpu::paged_summary(keys.data(), L, D, wp, out_dim, page);
                }
                py::array_t<float> a({(py::ssize_t)(flat.size() / out_dim), (py::ssize_t)out_dim});
                std::copy(flat.begin(), flat.end(), a.mutable_data());
                return a;
            }
        }
    }
    data_type::KVCacheData<float> raw = kv_of(retrieved_data);
    const int page = kw_required<int>(kwargs, "page_size", "PagedKVIndexBuilder");
    std::vector<std::vector<float>> w;
    if (kwargs.contains("weight") && !kwargs["weight"].is_none()) {
        w = rows_of(kwargs["weight"], "weight");
    } else {   // no projection: the identity (1.0 * x + 0 * y is exact)
        const size_t d = raw.get_head_dim();
        w.assign(d, std::vector<float>(d, 0.0f));
        for (size_t i = 0; i < d; ++i) w[i][i] = 1.0f;
    }
    data_type::FlatIndexMemory<float> out;
    {
        py::gil_scoped_release nogil;
        step::PagedKVIndexBuilder s(w, page);
        s.set_current_kernel(kt);
        s.execute(raw, out);
    }
    return to_array(out.export_data());
}

py::array_t<float> block_sparse(KernelType kt, const py::object& query,
                                const py::object& retrieved_data, const py::object& indices,
                                const py::object& input_data, const py::kwargs& kwargs) {
    // the attended vector: input_data when given, else the query
    const py::object& src = input_data.is_none() ? query : input_data;
    if (kt == KernelType::GPU) {
        const std::vector<float> q = vec_of(src, "input_data");
        const std::vector<int> blocks = ints_of(indices, "indices");
        const size_t page = kw_required<size_t>(kwargs, "page_size", "BlockSparseAttention");
        F32 keys, vals;
        if (matrix_with_cols(kv_part(retrieved_data, "keys", 0), q.size(), keys) &&
            matrix_with_cols(kv_part(retrieved_data, "values", 1), q.size(), vals) &&
            keys.shape(0) == vals.shape(0) && keys.shape(0) > 0 && !q.empty() &&
            !blocks.empty() && page > 0) {
            std::vector<float> out;
            {
                py::gil_scoped_release nogil;
                out = gpu::block_sparse_attention(keys.data(), vals.data(), (size_t)keys.shape(0),
                                                  q.size(), q.data(), blocks.data(), blocks.size(),
                                                  page);
            }
            return to_array(out);
        }
    }
    data_type::KVCacheData<float> raw = kv_of(retrieved_data);
    data_type::TopKIndex idx(ints_of(indices, "indices"));
    data_type::VectorInputOutputData<float> in(vec_of(src, "input_data"));
    const size_t page = kw_required<size_t>(kwargs, "page_size", "BlockSparseAttention");
    data_type::VectorInputOutputData<float> out;
    {
        py::gil_scoped_release nogil;
        step::BlockSparseAttention s(page);
        s.set_current_kernel(kt);
        s.execute(raw, idx, in, out);
    }
    return to_array(out.export_data());
}

py::array_t<int> bm25(KernelType kt, const py::object& memory, const py::object& query,
                      const py::kwargs&) {
    data_type::BM25IndexMemory mem = bm25_of(memory);
    data_type::BM25Query q = bm25_query_of(query);
    data_type::TopKIndex out;
    {
        py::gil_scoped_release nogil;
        step::FusedBM25Retrieval s;
        s.set_kernel(kt);
        s.execute(mem, q, out);
    }
    return to_array(out.export_data());
}

template <typename Fn>
void def_both(py::module_& m, const std::string& name, Fn fn, const char* doc) {
    for (const auto& kt : {std::make_pair(std::string("cpu"), KernelType::CPU),
                           std::make_pair(std::string("gpu"), KernelType::GPU)}) {
        const KernelType t = kt.second;
        m.def((name + "_" + kt.first).c_str(),
              [fn, t](py::args args, py::kwargs kwargs) { return fn(t, args, kwargs); }, doc);
    }
}

py::object arg(const py::args& args, size_t i, const char* fn, const char* what) {
    if (args.size() <= i)
        throw py::type_error(std::string(fn) + ": missing positional argument '" + what + "'");
    return args[i];
}

}  // namespace

PYBIND11_MODULE(heteromm_cpp_kernels, m) {
    m.doc() =
        "C++ step kernels of heteromm-b200 under the names the reference's pipeline "
        "generator calls: <StepClass>_cpu / <StepClass>_gpu.";
    def_both(m, "InnerProductCompute",
             [](KernelType t, py::args a, py::kwargs k) {
                 return py::object(inner_product(t, arg(a, 0, "InnerProductCompute", "memory"),
                                                 arg(a, 1, "InnerProductCompute", "query"), k));
             },
             "(memory [N, d] float32, query [d]) -> scores [N]: fp32 inner products, "
             "summed in index order.");
    def_both(m, "TopKRetrieval",
             [](KernelType t, py::args a, py::kwargs k) {
                 return py::object(topk(t, arg(a, 0, "TopKRetrieval", "scores"), k));
             },
             "(scores [N], k=64) -> indices of the min(k, N) best scores, best first, "
             "ties to the lowest index.");
    def_both(m, "ThresholdRetrieval",
             [](KernelType t, py::args a, py::kwargs k) {
                 return py::object(threshold(t, arg(a, 0, "ThresholdRetrieval", "scores"), k));
             },
             "(scores [N], threshold=T) -> ascending indices with score >= T.");
    def_both(m, "InnerProductTopKRetrieval",
             [](KernelType t, py::args a, py::kwargs k) {
                 return py::object(ip_topk(t, arg(a, 0, "InnerProductTopKRetrieval", "memory"),
                                           arg(a, 1, "InnerProductTopKRetrieval", "query"), k));
             },
             "(memory [N, d], query [d], k=64) -> top-k row indices of the inner products.");
    def_both(m, "PagedKVIndexBuilder",
             [](KernelType t, py::args a, py::kwargs k) {
                 return py::object(paged_builder(t, arg(a, 0, "PagedKVIndexBuilder", "retrieved_data"), k));
             },
             "((keys [L, D], values [L, D]), page_size=P, weight=[out, D] or None) -> "
             "page summaries [ceil(L/P), out]: fp32 token means, projected.");
    def_both(m, "BlockSparseAttention",
             [](KernelType t, py::args a, py::kwargs k) {
                 return py::object(block_sparse(
                     t, arg(a, 0, "BlockSparseAttention", "query"),
                     arg(a, 1, "BlockSparseAttention", "retrieved_data"),
                     arg(a, 2, "BlockSparseAttention", "indices"),
                     a.size() > 3 ? py::object(a[3]) : py::object(py::none()), k));
             },
             "(query [D], (keys, values), block indices, input_data [D] or None, page_size=P) "
             "-> attention output [D] over the selected blocks' tokens.");
    def_both(m, "FusedBM25Retrieval",
             [](KernelType t, py::args a, py::kwargs k) {
                 return py::object(bm25(t, arg(a, 0, "FusedBM25Retrieval", "memory"),
                                        arg(a, 1, "FusedBM25Retrieval", "query"), k));
             },
             "(documents: sequence of {token: tf}, query: {token: freq} or token ids) -> "
             "top-64 document indices by BM25 (k1 = 1.2, b = 0.75).");
}
