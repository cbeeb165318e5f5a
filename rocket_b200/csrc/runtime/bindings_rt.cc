// pybind11 bindings of the host runtime (no torch dependency).
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <pybind11/numpy.h>

#include "kv_manager.h"

namespace py = pybind11;
using namespace rkt_rt;

PYBIND11_MODULE(_rt, m) {
  m.doc() = "rocket_b200 host runtime: paged KV manager with radix prefix sharing";
  py::class_<CopyOp>(m, "CopyOp").def_readonly("src", &CopyOp::src).def_readonly("dst", &CopyOp::dst);
  py::class_<KvManager>(m, "KvManager")
      .def(py::init<int, int, int, bool>(), py::arg("num_pages"), py::arg("page_size"), py::arg("max_pages_per_seq"),
           py::arg("prefix_cache") = true)
      .def("open", &KvManager::open)
      .def("append", &KvManager::append)
      .def("truncate", &KvManager::truncate)
      .def("fork", &KvManager::fork)
      .def("free", &KvManager::free)
      .def("commit_prefix", &KvManager::commit_prefix)
      .def("length", &KvManager::length)
      .def("pages", &KvManager::pages)
      .def("can_append", &KvManager::can_append)
      .def("pages_needed", &KvManager::pages_needed)
      .def("num_free_pages", &KvManager::num_free_pages)
      .def("num_pages", &KvManager::num_pages)
      .def("page_size", &KvManager::page_size)
      .def("num_seqs", &KvManager::num_seqs)
      .def("cached_blocks", &KvManager::cached_blocks)
      .def("hits", &KvManager::hits)
      .def("lookups", &KvManager::lookups)
      .def("block_table",
           [](const KvManager& k, const std::vector<int64_t>& seqs, py::array_t<int32_t> out) {
             auto buf = out.mutable_unchecked<2>();
             if ((size_t)buf.shape(0) < seqs.size()) throw std::invalid_argument("block_table: too few rows");
             k.block_table(seqs, out.mutable_data(), (int)buf.shape(1));
           });
  m.def("block_key", [](uint64_t parent, const std::vector<int32_t>& toks) {
    return PrefixTree::block_key(parent, toks.data(), (int)toks.size());
  });
}
