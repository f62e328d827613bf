// Python bindings of the C++ runtime (module kapsl_sdk_b200._native):
// bincode wire codec, paged-KV block allocator, shared-memory transport and
// the socket / SHM servers.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "block_alloc.h"
#include "cpu_kernels.h"
#include "hnsw.h"
#include "server.h"
#include "shm.h"
#include "text_index.h"
#include "wasm.h"
#include "work_queue.h"
#include "wire.h"

namespace py = pybind11;
using namespace kapsl;

namespace {

template <class T>
std::optional<T> opt_get(const py::dict& d, const char* k) {
  if (!d.contains(k)) return std::nullopt;
  py::object v = d[k];
  if (v.is_none()) return std::nullopt;
  return v.cast<T>();
}

wire::Metadata metadata_from_py(const py::dict& d) {
  wire::Metadata m;
  m.request_id = opt_get<std::string>(d, "request_id");
  m.timeout_ms = opt_get<uint64_t>(d, "timeout_ms");
  if (auto p = opt_get<int>(d, "priority")) m.priority = (uint8_t)*p;
  m.force_cpu = opt_get<bool>(d, "force_cpu");
  m.model_version = opt_get<std::string>(d, "model_version");
  m.auth_token = opt_get<std::string>(d, "auth_token");
  m.max_new_tokens = opt_get<uint32_t>(d, "max_new_tokens");
  m.temperature = opt_get<float>(d, "temperature");
  m.top_p = opt_get<float>(d, "top_p");
  m.top_k = opt_get<uint32_t>(d, "top_k");
  m.repetition_penalty = opt_get<float>(d, "repetition_penalty");
  m.seed = opt_get<uint64_t>(d, "seed");
  m.stop_token_ids = opt_get<std::vector<uint32_t>>(d, "stop_token_ids");
  return m;
}

wire::Request request_from_py(const py::dict& d) {
  wire::Request r;
  r.input = packet_from_py(d["input"]);
  if (d.contains("additional_inputs") && !d["additional_inputs"].is_none())
    for (auto item : d["additional_inputs"]) {
      py::tuple t = item.cast<py::tuple>();
      r.additional_inputs.push_back({t[0].cast<std::string>(), packet_from_py(t[1])});
    }
  r.session_id = opt_get<std::string>(d, "session_id");
  if (d.contains("metadata") && !d["metadata"].is_none()) r.metadata = metadata_from_py(d["metadata"].cast<py::dict>());
  return r;
}

py::dict hybrid_req_to_py(const wire::HybridRequest& h) {
  py::dict d;
  d["request_id"] = h.meta.request_id;
  d["model_id"] = h.meta.model_id;
  d["priority"] = h.meta.priority;
  d["force_cpu"] = (bool)h.meta.force_cpu;
  d["timestamp_ns"] = h.meta.timestamp_ns;
  d["shm_offset"] = h.shm_offset;
  d["shm_size"] = h.shm_size;
  return d;
}

}  // namespace

namespace {
using F32 = py::array_t<float, py::array::c_style>;
using I64 = py::array_t<int64_t, py::array::c_style>;
using I32 = py::array_t<int32_t, py::array::c_style>;

void need(bool ok, const char* msg) {
  if (!ok) throw std::invalid_argument(msg);
}

void cpu_module(py::module_& m) {
  auto c = m.def_submodule("cpu", "fp32 CPU kernels of the CPU backend");
  c.def("rmsnorm", [](F32 x, F32 w, F32 out, float eps) {
    need(x.ndim() == 2 && out.size() == x.size() && w.size() == x.shape(1), "rmsnorm: x [T, d], w [d], out like x");
    py::gil_scoped_release nogil;
    kapsl::cpu::rmsnorm(x.data(), w.data(), out.mutable_data(), x.shape(0), x.shape(1), eps);
  });
  c.def("rope", [](F32 x, I64 pos, F32 cos_sin) {
    need(x.ndim() == 3 && pos.size() == x.shape(0) && cos_sin.ndim() == 2 && cos_sin.shape(1) == x.shape(2),
         "rope: x [T, H, D], positions [T], cos_sin [max_pos, D]");
    py::gil_scoped_release nogil;
    kapsl::cpu::rope(x.mutable_data(), pos.data(), cos_sin.data(), x.shape(0), x.shape(1), x.shape(2));
  });
  c.def("kv_write", [](F32 k, F32 v, I64 slots, F32 kc, F32 vc) {
    need(k.ndim() == 3 && kc.ndim() == 4 && kc.shape(1) == k.shape(1) && kc.shape(3) == k.shape(2) &&
             slots.size() == k.shape(0) && v.size() == k.size() && vc.size() == kc.size(),
         "kv_write: k/v [T, Hkv, D], caches [blocks, Hkv, bs, D]");
    py::gil_scoped_release nogil;
    kapsl::cpu::kv_write(k.data(), v.data(), slots.data(), kc.mutable_data(), vc.mutable_data(), k.shape(0),
                         k.shape(1), kc.shape(2), k.shape(2));
  });
  c.def("paged_attention", [](F32 q, F32 kc, F32 vc, I64 row0, I64 nq, I64 ctx, I32 bt, float scale, F32 out) {
    need(q.ndim() == 3 && kc.ndim() == 4 && bt.ndim() == 2 && out.size() == q.size() && q.shape(2) <= 512,
         "paged_attention: shapes (head_dim <= 512)");
    need(row0.size() == nq.size() && nq.size() == ctx.size() && bt.shape(0) >= row0.size(),
         "paged_attention: per-sequence arrays differ");
    py::gil_scoped_release nogil;
    kapsl::cpu::paged_attention(q.data(), kc.data(), vc.data(), row0.data(), nq.data(), ctx.data(), bt.data(),
                                bt.shape(1), row0.size(), q.shape(1), kc.shape(1), kc.shape(2), q.shape(2), scale,
                                out.mutable_data());
  });
  using U8 = py::array_t<uint8_t, py::array::c_style>;
  c.def("q4k_matmul", [](F32 x, U8 w, F32 y) {
    need(x.ndim() == 2 && w.ndim() == 2 && y.ndim() == 2, "q4k_matmul: x [T, K], w [N, K/256*144], y [T, N]");
    const int64_t T = x.shape(0), K = x.shape(1), N = w.shape(0);
    need(K % 256 == 0 && w.shape(1) == K / 256 * 144 && y.shape(0) == T && y.shape(1) == N, "q4k_matmul: shapes");
    py::gil_scoped_release nogil;
    kapsl::cpu::q4k_matmul(x.data(), w.data(), y.mutable_data(), T, N, K);
  });
  c.def("q4k_matmul_q8", [](F32 x, U8 w, F32 y) {
    need(x.ndim() == 2 && w.ndim() == 2 && y.ndim() == 2, "q4k_matmul_q8: x [T, K], w [N, K/256*144], y [T, N]");
    const int64_t T = x.shape(0), K = x.shape(1), N = w.shape(0);
    need(K % 256 == 0 && w.shape(1) == K / 256 * 144 && y.shape(0) == T && y.shape(1) == N, "q4k_matmul_q8: shapes");
    py::gil_scoped_release nogil;
    kapsl::cpu::q4k_matmul_q8(x.data(), w.data(), y.mutable_data(), T, N, K);
  });
  c.def("q6k_matmul_q8", [](F32 x, U8 w, F32 y) {
    need(x.ndim() == 2 && w.ndim() == 2 && y.ndim() == 2, "q6k_matmul_q8: x [T, K], w [N, K/256*210], y [T, N]");
    const int64_t T = x.shape(0), K = x.shape(1), N = w.shape(0);
    need(K % 256 == 0 && w.shape(1) == K / 256 * 210 && y.shape(0) == T && y.shape(1) == N, "q6k_matmul_q8: shapes");
    py::gil_scoped_release nogil;
    kapsl::cpu::q6k_matmul_q8(x.data(), w.data(), y.mutable_data(), T, N, K);
  });
  c.def("q6k_dequant_rows", [](U8 w, int64_t n0, int64_t n1, F32 out) {
    need(w.ndim() == 2 && 0 <= n0 && n0 <= n1 && n1 <= w.shape(0), "q6k_dequant_rows: rows");
    const int64_t K = w.shape(1) / 210 * 256;
    need(w.shape(1) % 210 == 0 && out.ndim() == 2 && out.shape(0) == n1 - n0 && out.shape(1) == K,
         "q6k_dequant_rows: out [n1 - n0, K]");
    py::gil_scoped_release nogil;
    kapsl::cpu::q6k_dequant_rows(w.data(), out.mutable_data(), n0, n1, K);
  });
  c.def("q80_matmul_q8", [](F32 x, U8 w, F32 y) {
    need(x.ndim() == 2 && w.ndim() == 2 && y.ndim() == 2, "q80_matmul_q8: x [T, K], w [N, K/32*34], y [T, N]");
    const int64_t T = x.shape(0), K = x.shape(1), N = w.shape(0);
    need(K % 256 == 0 && w.shape(1) == K / 32 * 34 && y.shape(0) == T && y.shape(1) == N, "q80_matmul_q8: shapes");
    py::gil_scoped_release nogil;
    kapsl::cpu::q80_matmul_q8(x.data(), w.data(), y.mutable_data(), T, N, K);
  });
  c.def("q80_dequant_rows", [](U8 w, int64_t n0, int64_t n1, F32 out) {
    need(w.ndim() == 2 && 0 <= n0 && n0 <= n1 && n1 <= w.shape(0), "q80_dequant_rows: rows");
    const int64_t K = w.shape(1) / 34 * 32;
    need(w.shape(1) % 34 == 0 && out.ndim() == 2 && out.shape(0) == n1 - n0 && out.shape(1) == K,
         "q80_dequant_rows: out [n1 - n0, K]");
    py::gil_scoped_release nogil;
    kapsl::cpu::q80_dequant_rows(w.data(), out.mutable_data(), n0, n1, K);
  });
  c.def("q4k_dequant_rows", [](U8 w, int64_t n0, int64_t n1, F32 out) {
    need(w.ndim() == 2 && 0 <= n0 && n0 <= n1 && n1 <= w.shape(0), "q4k_dequant_rows: rows");
    const int64_t K = w.shape(1) / 144 * 256;
    need(out.ndim() == 2 && out.shape(0) == n1 - n0 && out.shape(1) == K, "q4k_dequant_rows: out [n1 - n0, K]");
    py::gil_scoped_release nogil;
    kapsl::cpu::q4k_dequant_rows(w.data(), out.mutable_data(), n0, n1, K);
  });
  c.def("silu_mul", [](F32 x, F32 out) {
    need(x.ndim() == 2 && x.shape(1) % 2 == 0 && out.size() == x.size() / 2, "silu_mul: x [T, 2F], out [T, F]");
    py::gil_scoped_release nogil;
    kapsl::cpu::silu_mul(x.data(), out.mutable_data(), x.shape(0), x.shape(1) / 2);
  });
}
}  // namespace

PYBIND11_MODULE(_native, m) {
  cpu_module(m);
  m.doc() = "kapsl_sdk_b200 C++ runtime: wire codec, block allocator, SHM transport, servers";

  static py::object out_of_blocks;  // Python class kapsl_sdk_b200.llm.block_manager.OutOfBlocks
  py::register_exception_translator([](std::exception_ptr p) {
    try {
      if (p) std::rethrow_exception(p);
    } catch (const OutOfBlocksError& e) {
      if (!out_of_blocks) out_of_blocks = py::module_::import("kapsl_sdk_b200.llm.block_manager").attr("OutOfBlocks");
      PyErr_SetString(out_of_blocks.ptr(), e.what());
    } catch (const wire::DecodeError& e) {
      PyErr_SetString(PyExc_ValueError, e.what());
    } catch (const wasm::LoadError& e) {
      PyErr_SetString(PyExc_ValueError, (std::string("wasm module rejected: ") + e.what()).c_str());
    } catch (const wasm::Trap& e) {
      PyErr_SetString(PyExc_RuntimeError, (std::string("wasm trap: ") + e.what()).c_str());
    }
  });

  // ---- text indexing: suffix arrays and Unigram lattices (tokenizer training)
  auto tx = m.def_submodule("text", "suffix arrays, repeated substrings and Unigram lattices");
  tx.def("suffix_array", [](const std::u32string& s) {
    return text::suffix_array(std::vector<int32_t>(s.begin(), s.end()));
  }, "Start offsets of the suffixes of a string (code points) in lexicographic order");
  tx.def("lcp_array", [](const std::u32string& s) {
    const std::vector<int32_t> v(s.begin(), s.end());
    return text::lcp_array(v, text::suffix_array(v));
  });
  tx.def("repeated_substrings", [](const std::u32string& s) {
    std::vector<text::SubstringNode> nodes;
    {
      py::gil_scoped_release nogil;
      nodes = text::repeated_substrings(std::vector<int32_t>(s.begin(), s.end()));
    }
    py::list out;
    for (const auto& nd : nodes) out.append(py::make_tuple(s.substr(nd.offset, nd.length), nd.freq));
    return out;
  }, "Internal nodes of the suffix tree as (substring, occurrences), bottom-up, root (\"\") last");
  tx.def("top_repeated_substrings", [](const std::u32string& s, int32_t max_len, size_t limit,
                                      const std::u32string& banned, const std::u32string& not_inner) {
    std::vector<text::SubstringNode> nodes;
    {
      py::gil_scoped_release nogil;
      nodes = text::top_repeated_substrings(std::vector<int32_t>(s.begin(), s.end()), max_len, limit,
                                            std::vector<int32_t>(banned.begin(), banned.end()),
                                            std::vector<int32_t>(not_inner.begin(), not_inner.end()));
    }
    py::list out;
    for (const auto& nd : nodes) out.append(py::make_tuple(s.substr(nd.offset, nd.length), nd.freq));
    return out;
  }, py::arg("text"), py::arg("max_len"), py::arg("limit"), py::arg("banned") = std::u32string(),
     py::arg("not_inner") = std::u32string(),
     "Repeated substrings of 2..max_len code points with the largest occurrences * length, best first");
  py::class_<text::UnigramModel>(tx, "UnigramModel")
      .def(py::init<const std::vector<std::u32string>&, const std::vector<double>&, int>(), py::arg("pieces"),
           py::arg("scores"), py::arg("unk_id") = -1)
      .def("encode", &text::UnigramModel::encode, py::call_guard<py::gil_scoped_release>())
      .def("encode_batch", [](const text::UnigramModel& u, const std::vector<std::u32string>& texts) {
        std::vector<std::vector<int32_t>> out(texts.size());
        py::gil_scoped_release nogil;
        for (size_t i = 0; i < texts.size(); ++i) out[i] = u.encode(texts[i]);
        return out;
      })
      .def("expected_counts", [](const text::UnigramModel& u, const std::vector<std::u32string>& words,
                                 const std::vector<double>& freqs) {
        std::vector<double> counts;
        double ll;
        {
          py::gil_scoped_release nogil;
          ll = u.expected_counts(words, freqs, counts);
        }
        return py::make_tuple(counts, ll);
      }, "(expected count of every piece, sum of freq * log Z) over the words")
      .def("alternative", &text::UnigramModel::alternative)
      .def("alternative_scores", &text::UnigramModel::alternative_scores, py::call_guard<py::gil_scoped_release>())
      .def("__len__", &text::UnigramModel::size);

  // ---- RAG: approximate nearest-neighbour index (cosine)
  auto rg = m.def_submodule("rag", "vector index of the RAG store");
  py::class_<rag::Hnsw>(rg, "Hnsw")
      .def(py::init<int, int, int, uint64_t>(), py::arg("dim"), py::arg("M") = 16, py::arg("ef_construction") = 200,
           py::arg("seed") = 42)
      .def("add", [](rag::Hnsw& h, py::array_t<float, py::array::c_style | py::array::forcecast> x, int threads) {
        if (x.ndim() < 1 || x.ndim() > 2 || x.shape(x.ndim() - 1) != h.dim())
          throw std::invalid_argument("hnsw.add: expected [dim] or [n, dim] float32");
        const int64_t n = x.ndim() == 1 ? 1 : x.shape(0);
        py::array_t<int64_t> labels(n);
        auto L = labels.mutable_unchecked<1>();
        const float* p = x.data();
        {
          py::gil_scoped_release nogil;
          const int64_t first = n == 1 ? h.add(p) : h.add_batch(p, n, threads);
          for (int64_t i = 0; i < n; ++i) L(i) = first + i;
        }
        return labels;
      }, py::arg("vectors"), py::arg("threads") = 0,
         "Insert vectors (several at once: `threads` workers, 0 = one per core); returns their labels "
         "(0, 1, 2, ... in insertion order)")
      .def("remove", &rag::Hnsw::remove)
      .def("search", [](const rag::Hnsw& h, py::array_t<float, py::array::c_style | py::array::forcecast> q, int k,
                        int ef, py::object allowed) {
        if (q.size() != h.dim()) throw std::invalid_argument("hnsw.search: query has the wrong dimension");
        py::array_t<uint8_t, py::array::c_style | py::array::forcecast> mask;
        const uint8_t* mp = nullptr;
        int64_t ml = 0;
        if (!allowed.is_none()) {
          mask = allowed.cast<py::array_t<uint8_t, py::array::c_style | py::array::forcecast>>();
          mp = mask.data();
          ml = mask.size();
        }
        std::vector<std::pair<float, int64_t>> r;
        {
          py::gil_scoped_release nogil;
          r = h.search(q.data(), k, ef, mp, ml);
        }
        py::array_t<float> sc((py::ssize_t)r.size());
        py::array_t<int64_t> lb((py::ssize_t)r.size());
        for (size_t i = 0; i < r.size(); ++i) {
          sc.mutable_at(i) = r[i].first;
          lb.mutable_at(i) = r[i].second;
        }
        return py::make_tuple(sc, lb);
      }, py::arg("query"), py::arg("k"), py::arg("ef") = 64, py::arg("allowed") = py::none(),
         "(cosine similarities, labels), best first; `allowed` is a uint8 mask over labels")
      .def("__len__", &rag::Hnsw::size)
      .def_property_readonly("dim", &rag::Hnsw::dim)
      .def("save", &rag::Hnsw::save, py::call_guard<py::gil_scoped_release>())
      .def_static("load", &rag::Hnsw::load, py::call_guard<py::gil_scoped_release>());

  // ---- WebAssembly connectors (WASI preview1)
  m.def("wasm_run",
        [](py::bytes module, py::bytes stdin_data, std::vector<std::pair<std::string, std::string>> env,
           std::vector<std::tuple<std::string, std::string, bool>> preopens, uint64_t fuel, double timeout_s,
           size_t stdout_cap, size_t stderr_cap) {
          wasm::WasiConfig cfg;
          cfg.stdin_data = stdin_data;
          cfg.env = std::move(env);
          cfg.preopens = std::move(preopens);
          cfg.stdout_cap = stdout_cap;
          cfg.stderr_cap = stderr_cap;
          wasm::RunLimits lim;
          lim.fuel = fuel;
          lim.timeout_s = timeout_s;
          const std::string bytes = module;
          wasm::WasiResult res;
          {
            py::gil_scoped_release nogil;
            res = wasm::run_wasi(bytes, cfg, lim);
          }
          return py::make_tuple(res.exit_code, py::bytes(res.out), py::bytes(res.err));
        },
        py::arg("module"), py::arg("stdin") = py::bytes(), py::arg("env") = std::vector<std::pair<std::string, std::string>>{},
        py::arg("preopens") = std::vector<std::tuple<std::string, std::string, bool>>{},
        py::arg("fuel") = (uint64_t)4000000000ull, py::arg("timeout_s") = 30.0,
        py::arg("stdout_cap") = (size_t)4 << 20, py::arg("stderr_cap") = (size_t)256 << 10,
        "Run a WASI command module's _start once; returns (exit code, stdout, stderr)");
  m.def("wasm_call",
        [](py::bytes module, const std::string& name, py::list args, uint64_t fuel) {
          // instantiate a module without imports and call one export (values typed by its signature)
          const std::string bytes = module;
          wasm::RunLimits lim;
          lim.fuel = fuel;
          auto none = [](const std::string&, const std::string&, const wasm::FuncType&) { return wasm::HostFn{}; };
          wasm::Instance inst(wasm::Module::parse(bytes), none, lim);
          const uint32_t f = inst.export_func(name);
          const wasm::FuncType t = inst.type_of(f);
          if (args.size() != t.params.size()) throw std::invalid_argument("wrong number of arguments");
          std::vector<uint64_t> in;
          for (size_t i = 0; i < t.params.size(); ++i) {
            const uint8_t ty = t.params[i];
            if (ty == wasm::F32) {
              const float v = args[i].cast<float>();
              uint32_t u;
              std::memcpy(&u, &v, 4);
              in.push_back(u);
            } else if (ty == wasm::F64) {
              const double v = args[i].cast<double>();
              uint64_t u;
              std::memcpy(&u, &v, 8);
              in.push_back(u);
            } else if (ty == wasm::I32) {
              in.push_back((uint32_t)args[i].cast<int64_t>());
            } else {
              in.push_back((uint64_t)args[i].cast<int64_t>());
            }
          }
          std::vector<uint64_t> out;
          {
            py::gil_scoped_release nogil;
            out = inst.call(f, in);
          }
          py::list res;
          for (size_t i = 0; i < t.results.size(); ++i) {
            const uint8_t ty = t.results[i];
            if (ty == wasm::F32) {
              float v;
              const uint32_t u = (uint32_t)out[i];
              std::memcpy(&v, &u, 4);
              res.append(v);
            } else if (ty == wasm::F64) {
              double v;
              std::memcpy(&v, &out[i], 8);
              res.append(v);
            } else if (ty == wasm::I32) {
              res.append((int32_t)(uint32_t)out[i]);
            } else {
              res.append((int64_t)out[i]);
            }
          }
          return res;
        },
        py::arg("module"), py::arg("name"), py::arg("args") = py::list(), py::arg("fuel") = (uint64_t)1000000000ull,
        "Instantiate an import-free module and call one exported function");

  // ---- wire
  m.attr("OP_INFER") = wire::OP_INFER;
  m.attr("OP_INFER_STREAM") = wire::OP_INFER_STREAM;
  m.attr("OP_METRICS") = wire::OP_METRICS;
  m.attr("OP_HYBRID_INFER") = wire::OP_HYBRID_INFER;
  m.attr("STATUS_OK") = wire::STATUS_OK;
  m.attr("STATUS_ERR") = wire::STATUS_ERR;
  m.attr("STATUS_STREAM_CHUNK") = wire::STATUS_STREAM_CHUNK;
  m.attr("STATUS_STREAM_END") = wire::STATUS_STREAM_END;
  py::class_<WorkQueue>(m, "WorkQueue", "bounded scheduler queue: overflow policy, micro-batch take, depth")
      .def(py::init<size_t>(), py::arg("capacity"))
      .def("put", [](WorkQueue& q, py::object job, int policy, bool block) {
        PyObject* j = job.inc_ref().ptr();  // owned by the queue once accepted
        PyObject* dropped = nullptr;
        int r;
        {
          py::gil_scoped_release nogil;
          r = q.put(j, policy, block, &dropped);
        }
        if (r != WorkQueue::kAccepted) Py_DECREF(j);
        py::object d = dropped ? py::reinterpret_steal<py::object>(dropped) : py::object(py::none());
        return py::make_tuple(r == WorkQueue::kAccepted, d);
      }, py::arg("job"), py::arg("policy"), py::arg("block") = true,
         "policy 0 block, 1 drop newest, 2 drop oldest -> (accepted, evicted job or None)")
      .def("take", [](WorkQueue& q, size_t max_items, double delay_s) {
        std::vector<PyObject*> v;
        {
          py::gil_scoped_release nogil;
          v = q.take(max_items, delay_s);
        }
        py::list out;
        for (PyObject* p : v) out.append(py::reinterpret_steal<py::object>(p));
        return out;
      })
      .def("done", [](WorkQueue& q, size_t n) {
        py::gil_scoped_release nogil;
        q.done(n);
      })
      .def("close", [](WorkQueue& q) {
        py::gil_scoped_release nogil;
        q.close();
      })
      .def("depth", [](WorkQueue& q) {
        py::gil_scoped_release nogil;
        return q.depth();
      })
      .def_property_readonly("closed", [](WorkQueue& q) {
        py::gil_scoped_release nogil;
        return q.closed();
      })
      .def_property_readonly("capacity", &WorkQueue::capacity)
      .def("drain", [](WorkQueue& q) {
        std::vector<PyObject*> v;
        {
          py::gil_scoped_release nogil;
          v = q.drain();
        }
        py::list out;
        for (PyObject* p : v) out.append(py::reinterpret_steal<py::object>(p));
        return out;
      });
  py::class_<TokenChannel, std::shared_ptr<TokenChannel>>(m, "TokenChannel",
                                                          "token ids from the engine loop to a streaming connection")
      .def(py::init<>())
      .def("push", &TokenChannel::push)
      .def("finish", &TokenChannel::finish)
      .def("fail", &TokenChannel::fail)
      .def("cancel", &TokenChannel::cancel)
      .def("cancelled", &TokenChannel::cancelled)
      .def("pop", [](TokenChannel& c, int timeout_ms) {
        std::vector<int32_t> v;
        std::string e;
        int st;
        {
          py::gil_scoped_release nogil;
          st = c.pop(v, e, timeout_ms);
        }
        return py::make_tuple(st, v, e);
      }, "(status, tokens, error): status 0 tokens, 1 end, 2 error, 3 timeout");
  // One call per engine step: push tok[i] into chans[i], then close those with fin[i].
  m.def("push_tokens", [](const std::vector<std::shared_ptr<TokenChannel>>& chans, const std::vector<int32_t>& toks,
                          const std::vector<bool>& fin) {
    if (chans.size() != toks.size() || chans.size() != fin.size()) throw std::invalid_argument("push_tokens: lengths");
    py::gil_scoped_release nogil;
    std::vector<std::shared_ptr<TokenChannel>> wake;
    wake.reserve(chans.size());
    for (size_t i = 0; i < chans.size(); ++i) {
      chans[i]->push_quiet(toks[i], fin[i]);
      wake.push_back(chans[i]);
    }
    TokenNotifier::get().post(std::move(wake));  // the wakeups run off this thread
  });
  m.def("encode_packet", [](py::object shape, std::string dtype, py::bytes data) {
    return py::bytes(wire::encode_packet(packet_from_py(py::make_tuple(shape, dtype, data))));
  });
  m.def("decode_packet", [](py::bytes b) { return packet_to_py(wire::decode_packet(std::string(b))); });
  m.def("encode_request", [](py::dict d) { return py::bytes(wire::encode_request(request_from_py(d))); });
  m.def("decode_request", [](py::bytes b) { return request_to_py(wire::decode_request(std::string(b))); });
  m.def("encode_hybrid_request", [](py::dict d) {
    wire::HybridRequest h;
    h.meta.request_id = d["request_id"].cast<uint64_t>();
    h.meta.model_id = d["model_id"].cast<uint32_t>();
    h.meta.priority = opt_get<int>(d, "priority").value_or(0);
    h.meta.force_cpu = opt_get<bool>(d, "force_cpu").value_or(false) ? 1 : 0;
    h.meta.timestamp_ns = opt_get<uint64_t>(d, "timestamp_ns").value_or(0);
    h.shm_offset = d["shm_offset"].cast<uint64_t>();
    h.shm_size = d["shm_size"].cast<uint64_t>();
    return py::bytes(wire::encode_hybrid_request(h));
  });
  m.def("decode_hybrid_request", [](py::bytes b) { return hybrid_req_to_py(wire::decode_hybrid_request(b)); });
  m.def("decode_hybrid_response", [](py::bytes b) {
    auto h = wire::decode_hybrid_response(b);
    py::dict d;
    d["request_id"] = h.meta.request_id;
    d["status"] = h.meta.status;
    d["latency_ns"] = h.meta.latency_ns;
    d["shm_offset"] = h.shm_offset;
    d["shm_size"] = h.shm_size;
    return d;
  });
  m.def("request_header", [](uint32_t model, uint32_t op, uint32_t size) {
    return py::bytes(wire::request_header(model, op, size));
  });
  m.def("response_header", [](uint32_t st, uint32_t size) { return py::bytes(wire::response_header(st, size)); });
  m.def("validate_packet", [](py::object shape, std::string dtype, py::bytes data) {
    return wire::validate_packet(packet_from_py(py::make_tuple(shape, dtype, data)));
  });

  // ---- block allocator
  py::class_<BlockAllocator>(m, "BlockAllocator")
      .def(py::init<int64_t, int, bool, std::string>(), py::arg("num_blocks"), py::arg("block_size") = 16,
           py::arg("enable_prefix_cache") = true, py::arg("eviction") = "lru")
      .def_property_readonly("num_blocks", &BlockAllocator::num_blocks)
      .def_property_readonly("block_size", &BlockAllocator::block_size)
      .def_property_readonly("evicted_blocks", &BlockAllocator::evicted_blocks)
      .def("num_free", &BlockAllocator::num_free)
      .def("num_used", &BlockAllocator::num_used)
      .def("usage", &BlockAllocator::usage)
      .def("refcount", &BlockAllocator::refcount)
      .def("allocate", &BlockAllocator::allocate)
      .def("incref", &BlockAllocator::incref)
      .def("free", &BlockAllocator::free)
      .def("match_prefix", &BlockAllocator::match_prefix)
      .def("commit_prefix", &BlockAllocator::commit_prefix, py::arg("tokens"), py::arg("blocks"),
           py::arg("priority") = 0)
      .def("is_cached", &BlockAllocator::is_cached);

  // ---- shared memory
  py::class_<shm::Region>(m, "ShmRegion")
      .def_static("create", &shm::Region::create)
      .def_static("open", &shm::Region::open)
      .def_property_readonly("size", &shm::Region::size)
      .def_property_readonly("name", &shm::Region::name)
      .def("header", [](const shm::Region& r) {
        const auto& h = r.header();
        py::dict d;
        d["magic"] = h.magic;
        d["version"] = h.version;
        d["request_queue_offset"] = h.request_queue_offset;
        d["response_queue_offset"] = h.response_queue_offset;
        d["tensor_pool_offset"] = h.tensor_pool_offset;
        d["max_tensor_size"] = h.max_tensor_size;
        d["notify_read_fd"] = h.notify_read_fd;
        d["notify_write_fd"] = h.notify_write_fd;
        return d;
      })
      .def("write_tensor", [](shm::Region& r, uint64_t off, py::object shape, std::string dtype, py::bytes data) {
        shm::write_tensor(r, off, packet_from_py(py::make_tuple(shape, dtype, data)));
      })
      .def("read_tensor", [](const shm::Region& r, uint64_t off) { return packet_to_py(shm::read_tensor(r, off)); })
      .def("read_bytes", [](const shm::Region& r, uint64_t off, uint64_t n) {
        if (!r.in_bounds(off, n)) throw std::out_of_range("outside the region");
        return py::bytes(reinterpret_cast<const char*>(r.base() + off), n);
      })
      .def("init_rings", [](shm::Region& r) {
        shm::Ring<shm::ShmRequest>(r.base() + shm::REQ_RING_OFFSET, shm::RING_CAPACITY_ARG, true);
        shm::Ring<shm::ShmResponse>(r.base() + shm::RESP_RING_OFFSET, shm::RING_CAPACITY_ARG, true);
      })
      .def("push_request", [](shm::Region& r, uint64_t request_id, uint32_t model_id, int priority, uint64_t off,
                              uint64_t size) {
        shm::ShmRequest q{};
        q.meta.request_id = request_id;
        q.meta.model_id = model_id;
        q.meta.priority = (uint8_t)priority;
        q.tensor_offset = off;
        q.tensor_size = size;
        return shm::Ring<shm::ShmRequest>(r.base() + shm::REQ_RING_OFFSET, shm::RING_CAPACITY_ARG, false).push(q);
      })
      .def("pop_request", [](shm::Region& r) -> py::object {
        auto q = shm::Ring<shm::ShmRequest>(r.base() + shm::REQ_RING_OFFSET, shm::RING_CAPACITY_ARG, false).pop();
        if (!q) return py::none();
        return py::make_tuple(q->meta.request_id, q->meta.model_id, q->meta.priority, q->tensor_offset, q->tensor_size);
      })
      .def("pop_response", [](shm::Region& r) -> py::object {
        auto q = shm::Ring<shm::ShmResponse>(r.base() + shm::RESP_RING_OFFSET, shm::RING_CAPACITY_ARG, false).pop();
        if (!q) return py::none();
        return py::make_tuple(q->meta.request_id, q->meta.status, q->result_offset, q->result_size, q->error_offset);
      })
      .def("ring_len", [](shm::Region& r, bool responses) {
        return responses ? shm::Ring<shm::ShmResponse>(r.base() + shm::RESP_RING_OFFSET, shm::RING_CAPACITY_ARG, false).len()
                         : shm::Ring<shm::ShmRequest>(r.base() + shm::REQ_RING_OFFSET, shm::RING_CAPACITY_ARG, false).len();
      })
      .def("read_error", [](const shm::Region& r, uint64_t off) { return shm::read_error(r, off); })
      .def("mark_result_read", [](shm::Region& r, uint64_t off) { shm::mark_result_read(r, off); });

  py::class_<shm::TieredAllocator>(m, "TieredAllocator")
      .def(py::init<uint64_t, uint64_t, std::vector<uint64_t>, std::vector<uint32_t>, double>(), py::arg("base"),
           py::arg("pool_bytes"), py::arg("class_sizes") = std::vector<uint64_t>{},
           py::arg("weights") = std::vector<uint32_t>{}, py::arg("ttl_s") = 30.0)
      .def("try_allocate", &shm::TieredAllocator::try_allocate)
      .def("release", &shm::TieredAllocator::release)
      .def("in_use", &shm::TieredAllocator::in_use)
      .def("oldest_lease_ms", &shm::TieredAllocator::oldest_lease_ms)
      .def("largest_slot", &shm::TieredAllocator::largest_slot)
      .def("layout_summary", &shm::TieredAllocator::layout_summary);

  py::class_<shm::ModelPools>(m, "ModelPools")
      .def(py::init([](uint64_t base, uint64_t total_bytes, py::list models, double ttl_s) {
             // models: [(model_id, pool_bytes[, class_sizes[, weights]]), ...]
             std::vector<shm::ModelPoolSpec> specs;
             for (auto item : models) {
               auto t = item.cast<py::tuple>();
               shm::ModelPoolSpec s{t[0].cast<uint32_t>(), t[1].cast<uint64_t>(), {}, {}};
               if (t.size() > 2) s.class_sizes = t[2].cast<std::vector<uint64_t>>();
               if (t.size() > 3) s.weights = t[3].cast<std::vector<uint32_t>>();
               specs.push_back(std::move(s));
             }
             return std::make_unique<shm::ModelPools>(base, total_bytes, specs, ttl_s);
           }),
           py::arg("base"), py::arg("total_bytes"), py::arg("models"), py::arg("ttl_s") = 30.0)
      .def("try_allocate", &shm::ModelPools::try_allocate, py::arg("model_id"), py::arg("size"),
           py::arg("force") = false)
      .def("release", &shm::ModelPools::release)
      .def("has_pool", &shm::ModelPools::has_pool)
      .def("range", [](const shm::ModelPools& p, std::optional<uint32_t> id) { return p.range(id.value_or(UINT32_MAX)); },
           py::arg("model_id") = py::none())
      .def("usage", [](const shm::ModelPools& p, std::optional<uint32_t> id) {
             const shm::PoolUsage u = id ? p.model_usage(*id) : p.shared_usage();
             return py::make_tuple(u.in_use, u.oldest_lease_ms);
           }, py::arg("model_id") = py::none())
      .def("total_usage", [](const shm::ModelPools& p) {
        const shm::PoolUsage u = p.total_usage();
        return py::make_tuple(u.in_use, u.oldest_lease_ms);
      })
      .def("layout_summary", &shm::ModelPools::layout_summary)
      .def_static("plan", &shm::ModelPools::plan, py::arg("total_bytes"), py::arg("weights"), py::arg("reserve_pct") = 10,
                  py::arg("min_pool") = (uint64_t)64 << 10);

  // ---- servers
  py::class_<WireServer>(m, "WireServer")
      .def(py::init<py::object, std::optional<std::string>>(), py::arg("handler"), py::arg("auth_token") = py::none())
      .def("listen_unix", &WireServer::listen_unix)
      .def("listen_tcp", &WireServer::listen_tcp, py::arg("host") = "127.0.0.1", py::arg("port") = 9096)
      .def("attach_shm", &WireServer::attach_shm)
      .def("start", &WireServer::start)
      .def("stop", &WireServer::stop, py::call_guard<py::gil_scoped_release>())
      .def_property_readonly("running", &WireServer::running)
      .def_property_readonly("requests_served", &WireServer::requests_served);

  py::class_<ShmServer>(m, "ShmServer")
      .def(py::init<py::object, std::string, size_t, int, std::map<uint32_t, uint32_t>>(), py::arg("handler"),
           py::arg("name"), py::arg("size") = (size_t)256 << 20, py::arg("workers") = 4,
           py::arg("model_weights") = std::map<uint32_t, uint32_t>{})
      .def("pool_usage", [](const ShmServer& s, std::optional<uint32_t> id) -> py::tuple {
             const shm::PoolUsage u = !s.pools() ? shm::PoolUsage{}
                                      : id       ? s.pools()->model_usage(*id)
                                                 : s.pools()->shared_usage();
             return py::make_tuple(u.in_use, u.oldest_lease_ms);
           }, py::arg("model_id") = py::none())
      .def("pool_layout", [](const ShmServer& s) { return s.pools() ? s.pools()->layout_summary() : std::string(); })
      .def("start", &ShmServer::start)
      .def("stop", &ShmServer::stop, py::call_guard<py::gil_scoped_release>())
      .def_property_readonly("requests_served", &ShmServer::requests_served)
      .def_property_readonly("pool_in_use", &ShmServer::pool_in_use)
      .def_property_readonly("pool_oldest_lease_ms", &ShmServer::pool_oldest_lease_ms)
      .def_property_readonly("pool_exhausted", &ShmServer::pool_exhausted)
      .def_property_readonly("result_pool_base", &ShmServer::result_pool_base);
}
