// pybind11 bindings of the host runtime (no torch dependency).
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <pybind11/numpy.h>

#include <algorithm>
#include <memory>

#include "bpe.h"
#include "expert_balance.h"
#include "expert_cache.h"
#include "kv_manager.h"
#include "nvfp4_quant.h"
#include "prefix_store.h"
#include "safetensors.h"
#include "slab_io.h"
#include "stager.h"

namespace py = pybind11;
using namespace rkt_rt;

// Bytes of one tensor inside a mapped safetensors file, exposed through the buffer
// protocol; holds the file (and so the mapping) alive while any view exists.
struct TensorBytes {
  std::shared_ptr<SafetensorsFile> file;
  const uint8_t* ptr;
  size_t n;
};

PYBIND11_MODULE(_rt, m) {
  m.doc() = "rocket_b200 host runtime: paged KV manager, safetensors reader, BPE core";
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
      .def("block_keys", &KvManager::block_keys)
      .def("cached_prefix_blocks", &KvManager::cached_prefix_blocks)
      .def("import_block", &KvManager::import_block)
      .def("sealed_blocks", &KvManager::sealed_blocks)
      .def("prefix_cache", &KvManager::prefix_cache)
      .def("hits", &KvManager::hits)
      .def("lookups", &KvManager::lookups)
      .def("block_table",
           [](const KvManager& k, const std::vector<int64_t>& seqs, py::array out) {
             if (!out.dtype().is(py::dtype::of<int32_t>()) || !(out.flags() & py::array::c_style) || !out.writeable() ||
                 out.ndim() != 2)
               throw std::invalid_argument("block_table: out must be a writable C-contiguous 2-D int32 array");
             if ((size_t)out.shape(0) < seqs.size()) throw std::invalid_argument("block_table: too few rows");
             k.block_table(seqs, static_cast<int32_t*>(out.mutable_data()), (int)out.shape(1));
           });
  py::class_<TensorBytes>(m, "TensorBytes", py::buffer_protocol())
      .def_buffer([](TensorBytes& t) -> py::buffer_info {
        return py::buffer_info(const_cast<uint8_t*>(t.ptr), 1, py::format_descriptor<uint8_t>::format(), 1,
                               {(py::ssize_t)t.n}, {1}, /*readonly=*/true);
      })
      .def("__len__", [](const TensorBytes& t) { return t.n; });
  py::class_<SafetensorsFile, std::shared_ptr<SafetensorsFile>>(m, "SafetensorsFile")
      .def(py::init<const std::string&>())
      .def("keys", &SafetensorsFile::keys)
      .def("metadata", &SafetensorsFile::metadata)
      .def("file_size", &SafetensorsFile::file_size)
      .def("info",
           [](const SafetensorsFile& f, const std::string& name) {
             const TensorInfo& t = f.info(name);
             return py::make_tuple(t.dtype, t.shape, t.begin, t.end);
           })
      .def("bytes", [](std::shared_ptr<SafetensorsFile> f, const std::string& name) {
        const TensorInfo& t = f->info(name);
        return TensorBytes{f, f->data(name), (size_t)(t.end - t.begin)};
      });
  m.def("dtype_itemsize", &dtype_itemsize);
  // NVFP4 host codec + offline materializer
  m.def("e4m3_from_float", &e4m3_from_float);
  m.def("e4m3_to_float", &e4m3_to_float);
  m.def("quantize_nvfp4",
        [](py::buffer src, const std::string& dtype, int64_t rows, int64_t cols, float g, int threads) {
          py::buffer_info bi = src.request();
          const SrcType t = dtype == "F32" ? SrcType::F32 : dtype == "BF16" ? SrcType::BF16
                          : dtype == "F16" ? SrcType::F16 : throw std::invalid_argument("dtype: F32 | BF16 | F16");
          const int64_t isz = t == SrcType::F32 ? 4 : 2;
          if ((int64_t)(bi.size * bi.itemsize) < rows * cols * isz) throw std::invalid_argument("source too small");
          py::array_t<uint8_t> packed({rows, cols / 2}), sf({rows, cols / 16});
          float gs;
          {
            py::gil_scoped_release nogil;
            gs = quantize_nvfp4(bi.ptr, t, rows, cols, g, packed.mutable_data(), sf.mutable_data(), threads);
          }
          return py::make_tuple(packed, sf, gs);
        },
        py::arg("src"), py::arg("dtype"), py::arg("rows"), py::arg("cols"), py::arg("global_scale") = 0.f,
        py::arg("threads") = 0);
  m.def("swizzle_sf", [](py::array_t<uint8_t, py::array::c_style> sf) {
    if (sf.ndim() != 2) throw std::invalid_argument("swizzle_sf: [rows, K/16] scales");
    py::array_t<uint8_t> out((py::ssize_t)sf_swizzled_bytes(sf.shape(0), sf.shape(1)));
    swizzle_sf(sf.data(), sf.shape(0), sf.shape(1), out.mutable_data());
    return out;
  });
  m.def("materialize_nvfp4",
        [](const std::vector<std::string>& inputs, const std::string& out_dir, const std::set<std::string>& quantize,
           const std::set<std::string>& cast_bf16, uint64_t shard_bytes, int threads,
           const std::map<std::string, std::string>& meta, const std::set<std::string>& fp8_rows) {
          MaterializeOptions o;
          o.inputs = inputs;
          o.out_dir = out_dir;
          o.quantize = quantize;
          o.fp8_rows = fp8_rows;
          o.cast_bf16 = cast_bf16;
          o.shard_bytes = shard_bytes;
          o.threads = threads;
          o.meta = meta;
          MaterializeReport r;
          {
            py::gil_scoped_release nogil;
            r = materialize_nvfp4(o);
          }
          py::dict d;
          d["files"] = r.files;
          d["tensors_in"] = r.tensors_in;
          d["quantized"] = r.quantized;
          d["bytes_in"] = r.bytes_in;
          d["bytes_out"] = r.bytes_out;
          d["max_rel_err"] = r.max_rel_err;
          d["worst"] = r.worst;
          d["checksums"] = r.checksums;
          return d;
        },
        py::arg("inputs"), py::arg("out_dir"), py::arg("quantize"), py::arg("cast_bf16") = std::set<std::string>{},
        py::arg("shard_bytes") = 4ull << 30, py::arg("threads") = 0,
        py::arg("meta") = std::map<std::string, std::string>{}, py::arg("fp8_rows") = std::set<std::string>{});
  m.def("stage_step",
        [](KvManager& kv, const std::vector<std::tuple<int64_t, std::vector<int32_t>, int32_t, int32_t, int32_t,
                                                     int32_t, int32_t, std::vector<int32_t>>>& items,
           int B, int K, int tpb, int page_size, int dummy_page, int dummy_slot,
           const std::map<std::string, std::pair<int, int>>& layout, py::array meta, py::array bt, int pad_rows) {
          // written in place: refuse anything pybind would have to convert (a converted copy
          // would silently drop the writes)
          for (py::array* arr : {&meta, &bt})
            if (!arr->dtype().is(py::dtype::of<int32_t>()) || !(arr->flags() & py::array::c_style) ||
                !arr->writeable())
              throw std::invalid_argument("stage_step: meta / bt must be writable C-contiguous int32 arrays");
          std::vector<StageItem> v;
          v.reserve(items.size());
          for (auto& it : items) {
            StageItem s;
            s.rid = std::get<0>(it);
            s.tokens = std::get<1>(it);
            s.start = std::get<2>(it);
            s.sample = std::get<3>(it);
            s.verify = std::get<4>(it);
            s.reserve = std::get<5>(it);
            s.state_slot = std::get<6>(it);
            s.next_prompt = std::get<7>(it);
            v.push_back(std::move(s));
          }
          MetaLayout L;
          for (auto& kvp : layout)
            if (kvp.second.first < 0 || (py::ssize_t)kvp.second.first + kvp.second.second > meta.size())
              throw std::invalid_argument("stage_step: layout field " + kvp.first + " outside the buffer");
          auto get = [&](const char* k) {
            auto f = layout.find(k);
            return f == layout.end() ? -1 : f->second.first;
          };
          auto cap = [&](const char* k) {
            auto f = layout.find(k);
            return f == layout.end() ? 0 : f->second.second;
          };
          L.ids = get("ids"); L.pos = get("pos"); L.slots = get("slots"); L.q_start = get("q_start");
          L.q_len = get("q_len"); L.kv_len = get("kv_len"); L.w_seq = get("w_seq"); L.w_tok0 = get("w_tok0");
          L.num_work = get("num_work"); L.out_rows = get("out_rows"); L.state_slot = get("state_slot");
          L.verify = get("verify"); L.sample = get("sample"); L.out_idx = get("out_idx"); L.next_tok = get("next_tok");
          if (L.ids < 0 || L.pos < 0 || L.slots < 0 || L.q_start < 0 || L.q_len < 0 || L.kv_len < 0 || L.w_seq < 0 ||
              L.w_tok0 < 0 || L.num_work < 0 || L.out_rows < 0 || L.state_slot < 0)
            throw std::invalid_argument("stage_step: layout misses a field");
          if (bt.ndim() != 2 || bt.shape(0) < B) throw std::invalid_argument("stage_step: block table rows < B");
          L.max_tokens = std::min({cap("ids"), cap("pos"), cap("slots")});
          if (K) L.max_tokens = std::min({L.max_tokens, cap("out_idx"), cap("next_tok")});
          L.max_seqs = std::min({cap("q_start"), cap("q_len"), cap("kv_len"), cap("state_slot")});
          if (K) L.max_seqs = std::min({L.max_seqs, cap("verify"), cap("sample")});
          L.max_work = std::min(cap("w_seq"), cap("w_tok0"));
          L.max_out = cap("out_rows");
          StageOut o;
          {
            py::gil_scoped_release nogil;
            o = stage_step(kv, v, B, K, tpb, page_size, dummy_page, dummy_slot, L,
                           static_cast<int32_t*>(meta.mutable_data()), static_cast<int32_t*>(bt.mutable_data()),
                           (int)bt.shape(1), pad_rows);
          }
          return py::make_tuple(o.T, o.S, o.work, o.n_out);
        },
        py::arg("kv"), py::arg("items"), py::arg("B"), py::arg("K"), py::arg("tpb"), py::arg("page_size"),
        py::arg("dummy_page"), py::arg("dummy_slot"), py::arg("layout"), py::arg("meta"), py::arg("bt"),
        py::arg("pad_rows") = -1);
  py::class_<ExpertSlotCache>(m, "ExpertSlotCache")
      .def(py::init<int, int>(), py::arg("num_experts"), py::arg("num_slots"))
      .def("plan",
           [](ExpertSlotCache& c, const std::vector<int32_t>& needed) {
             py::list out;
             for (auto& p : c.plan(needed)) out.append(py::make_tuple(p.remap, p.loads));
             return out;
           })
      .def("slot_of", &ExpertSlotCache::slot_of)
      .def("expert_in", &ExpertSlotCache::expert_in)
      .def("reset", &ExpertSlotCache::reset)
      .def("num_slots", &ExpertSlotCache::num_slots)
      .def("num_experts", &ExpertSlotCache::num_experts)
      .def("stats", [](const ExpertSlotCache& c) {
        py::dict d;
        d["hits"] = c.hits();
        d["misses"] = c.misses();
        d["evictions"] = c.evictions();
        d["passes"] = c.passes();
        return d;
      });
  m.def("file_digest_hex", &file_digest_hex);
  m.def("digest_hex", [](py::buffer b) {
    py::buffer_info bi = b.request();
    return digest_hex(static_cast<const uint8_t*>(bi.ptr), (uint64_t)(bi.size * bi.itemsize));
  });
  py::class_<SlabReader>(m, "SlabReader")
      .def(py::init<const std::string&, int, bool>(), py::arg("path"), py::arg("threads") = 4,
           py::arg("direct") = true)
      .def("file_size", &SlabReader::file_size)
      .def("submit",
           [](SlabReader& r, uintptr_t dst, uint64_t off, uint64_t n,
              const std::vector<std::tuple<uint64_t, uint64_t, std::string>>& checks) {
             std::vector<SlotCheck> c;
             for (auto& t : checks) c.push_back({std::get<0>(t), std::get<1>(t), std::get<2>(t)});
             return r.submit(dst, off, n, std::move(c));
           },
           py::arg("dst"), py::arg("offset"), py::arg("n"),
           py::arg("checks") = std::vector<std::tuple<uint64_t, uint64_t, std::string>>{})
      .def("wait", &SlabReader::wait, py::call_guard<py::gil_scoped_release>())
      .def("bytes_read", &SlabReader::bytes_read)
      .def("direct_reads", &SlabReader::direct_reads);
  m.def("verify_checksums", &verify_checksums);
  py::class_<PrefixStore>(m, "PrefixStore")
      .def(py::init<const std::string&, uint64_t, uint64_t, bool>(), py::arg("dir"), py::arg("max_bytes"),
           py::arg("segment_bytes") = 256ull << 20, py::arg("direct_io") = false)
      .def("put",
           [](PrefixStore& s, uint64_t key, uint64_t fp, const std::vector<py::buffer>& parts) {
             std::vector<py::buffer_info> infos;
             std::vector<std::pair<const uint8_t*, size_t>> p;
             for (auto& b : parts) {
               infos.push_back(b.request());
               auto& i = infos.back();
               p.emplace_back(static_cast<const uint8_t*>(i.ptr), (size_t)(i.size * i.itemsize));
             }
             py::gil_scoped_release nogil;
             return s.put(key, fp, p);
           })
      .def("contains", &PrefixStore::contains)
      .def("sizes", &PrefixStore::sizes)
      .def("get_into",
           [](PrefixStore& s, uint64_t key, uint64_t fp, const std::vector<py::buffer>& outs) {
             std::vector<py::buffer_info> infos;
             std::vector<std::pair<uint8_t*, size_t>> p;
             for (auto& b : outs) {
               infos.push_back(b.request(true));
               auto& i = infos.back();
               p.emplace_back(static_cast<uint8_t*>(i.ptr), (size_t)(i.size * i.itemsize));
             }
             py::gil_scoped_release nogil;
             return s.get_into(key, fp, p);
           })
      .def("get",
           [](PrefixStore& s, uint64_t key, uint64_t fp) -> py::object {
             auto sz = s.sizes(key, fp);
             if (sz.empty()) {
               std::vector<std::pair<uint8_t*, size_t>> none;
               return py::none();
             }
             std::vector<std::string> bufs;
             std::vector<std::pair<uint8_t*, size_t>> p;
             for (auto n : sz) bufs.emplace_back((size_t)n, '\0');
             for (auto& b : bufs) p.emplace_back(reinterpret_cast<uint8_t*>(&b[0]), b.size());
             if (!s.get_into(key, fp, p)) return py::none();
             py::list out;
             for (auto& b : bufs) out.append(py::bytes(b));
             return out;
           })
      .def("erase", &PrefixStore::erase)
      .def("flush", &PrefixStore::flush)
      .def("stats", [](const PrefixStore& s) {
        auto t = s.stats();
        py::dict d;
        d["puts"] = t.puts;
        d["gets"] = t.gets;
        d["hits"] = t.hits;
        d["misses"] = t.misses;
        d["checksum_failures"] = t.checksum_failures;
        d["torn_tail_recoveries"] = t.torn_tail_recoveries;
        d["evicted_records"] = t.evicted_records;
        d["bytes_written"] = t.bytes_written;
        d["bytes_read"] = t.bytes_read;
        d["live_records"] = t.live_records;
        d["live_bytes"] = t.live_bytes;
        d["refused_low_space"] = t.refused_low_space;
        return d;
      })
      .def("set_min_free_bytes", &PrefixStore::set_min_free_bytes)
      .def("min_free_bytes", &PrefixStore::min_free_bytes);
  m.def("balance_experts", [](const std::vector<int64_t>& hist, int ranks) {
    ExpertPlacement p = balance_experts(hist, ranks);
    return py::make_tuple(p.owner, p.order, p.rank_load);
  });
  py::class_<BpeModel>(m, "BpeModel")
      .def(py::init<const std::vector<std::pair<std::string, int32_t>>&,
                    const std::vector<std::pair<std::string, std::string>>&, bool>())
      .def("encode_piece", [](BpeModel& b, const py::bytes& p) { return b.encode_piece(std::string(p)); })
      .def("encode_pieces", &BpeModel::encode_pieces)
      .def("decode", [](const BpeModel& b, const std::vector<int32_t>& ids) { return py::bytes(b.decode(ids)); })
      .def("token_id", [](const BpeModel& b, const py::bytes& p) { return b.token_id(std::string(p)); })
      .def("vocab_size", &BpeModel::vocab_size)
      .def("num_merges", &BpeModel::num_merges);
  m.def("block_key", [](uint64_t parent, const std::vector<int32_t>& toks) {
    return PrefixTree::block_key(parent, toks.data(), (int)toks.size());
  });
}
