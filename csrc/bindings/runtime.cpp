// runtime.cpp -- binding of the host runtime: Bootstrap (and, below, Runtime/Barrier/AM).
#include <torch/extension.h>

#include "gicc/bootstrap.hpp"
#include "gicc/runtime.hpp"

namespace py = pybind11;
using gicc::Bootstrap;

namespace {

py::bytes to_bytes(const std::vector<uint8_t>& v) { return py::bytes(reinterpret_cast<const char*>(v.data()), v.size()); }

}  // namespace

void bind_runtime_objects(py::module_& m);  // runtime_objects.cpp

namespace gicc {
namespace fake {
int barrier_run(uint64_t* shm, int rank, int size, int iters, int mode, uint64_t timeout_ns, int skip_at, int* fail_iter);
int barrier_run_inject(uint64_t* shm, int rank, int size, int iters, int mode, uint64_t timeout_ns, int skip_at,
                       int* fail_iter, int inject_mode, int inject_at);
size_t am_region_bytes(int size, int nslots, uint32_t slot_bytes);
int am_run(uint8_t* shm, int rank, int size, int nslots, int nmsg, int nreq, uint64_t timeout_ns, uint64_t* out_counter,
           uint64_t* out_checksum);
int am_wait_one(uint8_t* shm, int rank, int size, int nslots, int src, uint64_t timeout_ns);
int cmdring_selftest(int ncmds, int nslots, uint64_t idle_timeout_ns);
int litmus_run(uint64_t* shm, int rank, int test, int iters, int k, int use_fence, uint32_t seed, uint32_t max_delay,
               uint64_t timeout_ns, uint64_t* violations);
}  // namespace fake
}  // namespace gicc

void bind_runtime(py::module_& m) {
  py::register_exception<gicc::BootstrapError>(m, "BootstrapError", PyExc_RuntimeError);

  m.def("p2p_links", []() {
    py::list out;
    for (const auto& l : gicc::p2p_links()) {
      py::dict d;
      d["src"] = l.src;
      d["dst"] = l.dst;
      d["access"] = l.access;
      d["native_atomics"] = l.native_atomics;
      d["array_access"] = l.array_access;
      d["perf_rank"] = l.perf_rank;
      out.append(d);
    }
    return out;
  }, "cudaDeviceGetP2PAttribute for every ordered pair of visible GPUs");
  m.def("check_exchange_consistency", &gicc::check_exchange_consistency, py::arg("boot"), py::arg("kinds"),
        py::arg("multicast"), py::call_guard<py::gil_scoped_release>(),
        "exchange()'s collective check of the newly registered buffer tables (no GPU needed)");
  py::class_<Bootstrap, std::shared_ptr<Bootstrap>>(m, "Bootstrap")
      .def(py::init<>(), py::call_guard<py::gil_scoped_release>(), "bootstrap from the environment (blocks for all ranks)")
      .def(py::init<int, int, const std::string&, double>(), py::arg("rank"), py::arg("size"), py::arg("addr"),
           py::arg("timeout_s") = -1.0, py::call_guard<py::gil_scoped_release>())
      .def("setup", &Bootstrap::setup, py::arg("local_rank_hint") = -1, py::arg("local_size_hint") = -1,
           py::call_guard<py::gil_scoped_release>())
      .def_property_readonly("rank", &Bootstrap::rank)
      .def_property_readonly("size", &Bootstrap::size)
      .def_property_readonly("local_rank", &Bootstrap::local_rank)
      .def_property_readonly("local_size", &Bootstrap::local_size)
      .def_property_readonly("server_port", &Bootstrap::server_port)
      .def_property_readonly("job_id", &Bootstrap::job_id)
      .def_property_readonly("timeout_s", &Bootstrap::timeout_s)
      .def("locality_map", &Bootstrap::locality_map)
      .def("barrier", &Bootstrap::barrier, py::call_guard<py::gil_scoped_release>())
      .def("allgather",
           [](Bootstrap& b, py::bytes data) {
             std::string s = data;
             std::vector<std::vector<uint8_t>> all;
             {
               py::gil_scoped_release rel;
               all = b.allgather(s.data(), (int)s.size());
             }
             py::list out;
             for (auto& v : all) out.append(to_bytes(v));
             return out;
           })
      .def("broadcast",
           [](Bootstrap& b, py::object data, int root) {
             // root passes bytes; every rank receives them (length is broadcast first)
             std::string s;
             if (b.rank() == root) s = data.cast<std::string>();
             uint64_t len = s.size();
             {
               py::gil_scoped_release rel;
               b.broadcast(len, root);
               s.resize(len);
               b.broadcast_bytes(&s[0], len, root);
             }
             return py::bytes(s);
           },
           py::arg("data"), py::arg("root") = 0)
      .def("send",
           [](Bootstrap& b, py::bytes data, int dst, int tag) {
             std::string s = data;
             py::gil_scoped_release rel;
             b.send(s.data(), s.size(), dst, tag);
           },
           py::arg("data"), py::arg("dst"), py::arg("tag") = 0)
      .def("recv",
           [](Bootstrap& b, size_t n, int src, int tag) {
             std::string s(n, '\0');
             {
               py::gil_scoped_release rel;
               b.recv(&s[0], n, src, tag);
             }
             return py::bytes(s);
           },
           py::arg("nbytes"), py::arg("src"), py::arg("tag") = 0)
      .def("sendrecv",
           [](Bootstrap& b, py::bytes data, int dst, size_t n, int src, int tag) {
             std::string s = data;
             std::string r(n, '\0');
             {
               py::gil_scoped_release rel;
               b.sendrecv(s.data(), s.size(), dst, &r[0], n, src, tag);
             }
             return py::bytes(r);
           },
           py::arg("data"), py::arg("dst"), py::arg("nbytes"), py::arg("src"), py::arg("tag") = 0)
      .def("wtime", &Bootstrap::wtime)
      .def("kv_put",
           [](Bootstrap& b, const std::string& k, py::bytes v) {
             std::string s = v;
             py::gil_scoped_release rel;
             b.kv_put(k, s.data(), s.size());
           })
      .def("kv_get",
           [](Bootstrap& b, const std::string& k, int consume) {
             std::vector<uint8_t> v;
             {
               py::gil_scoped_release rel;
               v = b.kv_get(k, consume);
             }
             return to_bytes(v);
           },
           py::arg("key"), py::arg("consume") = 0)
      .def("check", &Bootstrap::check, py::call_guard<py::gil_scoped_release>())
      .def("fail_job", &Bootstrap::fail_job, py::call_guard<py::gil_scoped_release>())
      .def("abort_job", &Bootstrap::abort_job, py::call_guard<py::gil_scoped_release>())
      .def("send_fds", &Bootstrap::send_fds, py::call_guard<py::gil_scoped_release>())
      .def("recv_fds", &Bootstrap::recv_fds, py::call_guard<py::gil_scoped_release>());

  // CPU-rank protocol runners over shared memory (the same protocol code as the kernels)
  m.def("cpu_barrier_run", [](uint64_t shm, int rank, int size, int iters, int mode, uint64_t timeout_ns, int skip_at) {
    int fail = -1;
    int st;
    {
      py::gil_scoped_release rel;
      st = gicc::fake::barrier_run(reinterpret_cast<uint64_t*>(shm), rank, size, iters, mode, timeout_ns, skip_at, &fail);
    }
    return py::make_tuple(st, fail);
  });
  m.def("cpu_am_region_bytes", &gicc::fake::am_region_bytes);
  m.def("cpu_am_run", [](uint64_t shm, int rank, int size, int nslots, int nmsg, int nreq, uint64_t timeout_ns) {
    uint64_t c = 0, k = 0;
    int st;
    {
      py::gil_scoped_release rel;
      st = gicc::fake::am_run(reinterpret_cast<uint8_t*>(shm), rank, size, nslots, nmsg, nreq, timeout_ns, &c, &k);
    }
    return py::make_tuple(st, c, k);
  });
  m.def("cpu_barrier_run_inject", [](uint64_t shm, int rank, int size, int iters, int mode, uint64_t timeout_ns,
                                     int inject_mode, int inject_at) {
    int fail = -1, st;
    {
      py::gil_scoped_release nogil;
      st = gicc::fake::barrier_run_inject(reinterpret_cast<uint64_t*>(shm), rank, size, iters, mode, timeout_ns, -1,
                                          &fail, inject_mode, inject_at);
    }
    return py::make_tuple(st, fail);
  });
  m.def("cpu_cmdring_selftest", [](int ncmds, int nslots, uint64_t idle_timeout_ns) {
    py::gil_scoped_release nogil;
    return gicc::fake::cmdring_selftest(ncmds, nslots, idle_timeout_ns);
  });
  m.def("cpu_litmus_run", [](uint64_t shm, int rank, int test, int iters, int k, int use_fence, uint32_t seed,
                             uint32_t max_delay, uint64_t timeout_ns) {
    uint64_t v = 0;
    int st;
    {
      py::gil_scoped_release nogil;
      st = gicc::fake::litmus_run(reinterpret_cast<uint64_t*>(shm), rank, test, iters, k, use_fence, seed, max_delay,
                                  timeout_ns, &v);
    }
    return py::make_tuple(st, v);
  });
  m.def("cpu_am_wait_one", [](uint64_t shm, int rank, int size, int nslots, int src, uint64_t timeout_ns) {
    py::gil_scoped_release rel;
    return gicc::fake::am_wait_one(reinterpret_cast<uint8_t*>(shm), rank, size, nslots, src, timeout_ns);
  });
  bind_runtime_objects(m);
}
