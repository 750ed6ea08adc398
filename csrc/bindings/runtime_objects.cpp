// runtime_objects.cpp -- binding of Runtime, Barrier and the communication kernels.
// Device addresses cross the boundary as Python ints.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "gicc/cmdring.hpp"
#include "gicc/am.hpp"
#include "gicc/barrier.hpp"
#include "gicc/ops.hpp"
#include "gicc/runtime.hpp"

namespace py = pybind11;
using namespace gicc;

namespace {
cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }
template <class T>
T* P(uint64_t a) {
  return reinterpret_cast<T*>(static_cast<uintptr_t>(a));
}
uint64_t A(const void* p) { return static_cast<uint64_t>(reinterpret_cast<uintptr_t>(p)); }

py::dict buf_dict(const Buffer& b) {
  py::dict d;
  d["ptr"] = A(b.ptr);
  d["size"] = b.size;
  d["addr"] = b.addr;
  d["lkey"] = b.lkey;
  d["rkey"] = b.rkey;
  d["index"] = b.index;
  return d;
}
Buffer to_buf(Runtime& rt, int idx) { return rt.buffer(idx); }
}  // namespace

void bind_runtime_objects(py::module_& m) {
  py::class_<RuntimeOptions>(m, "RuntimeOptions")
      .def(py::init<>())
      .def_readwrite("device", &RuntimeOptions::device)
      .def_readwrite("signal_heap_bytes", &RuntimeOptions::signal_heap_bytes)
      .def_readwrite("enable_multicast", &RuntimeOptions::enable_multicast);

  py::class_<Runtime, std::shared_ptr<Runtime>>(m, "Runtime")
      .def(py::init<>(), py::call_guard<py::gil_scoped_release>())
      .def(py::init<std::shared_ptr<Bootstrap>, RuntimeOptions>(), py::arg("boot"), py::arg("options") = RuntimeOptions(),
           py::call_guard<py::gil_scoped_release>())
      .def("register_buffer",
           [](Runtime& r, uint64_t ptr, size_t size, bool is_device) {
             return buf_dict(r.register_buffer(P<void>(ptr), size, is_device));
           },
           py::arg("ptr"), py::arg("size"), py::arg("is_device") = true)
      .def("alloc", [](Runtime& r, size_t n, bool mc) { return buf_dict(r.alloc(n, mc)); }, py::arg("nbytes"),
           py::arg("multicast") = false)
      .def("exchange", &Runtime::exchange, py::call_guard<py::gil_scoped_release>())
      .def("remote_buffer",
           [](Runtime& r, int rank, int idx) {
             RemoteBufferInfo i = r.remote_buffer(rank, idx);
             return py::make_tuple(i.addr, i.rkey);
           })
      .def("remote_ptr", [](Runtime& r, int rank, int idx, size_t off) { return A(r.remote_ptr(rank, idx, off)); },
           py::arg("rank"), py::arg("buf_index"), py::arg("offset") = 0)
      .def("translate", [](Runtime& r, uint64_t local, int peer) { return A(r.translate(P<void>(local), peer)); })
      .def("multicast_ptr", [](Runtime& r, int idx) { return A(r.multicast_ptr(idx)); })
      .def_property_readonly("multicast_supported", &Runtime::multicast_supported)
      .def("buffer", [](Runtime& r, int idx) { return buf_dict(r.buffer(idx)); })
      .def_property_readonly("num_buffers", &Runtime::num_buffers)
      .def("prepare", [](Runtime& r, int peer, int idx) { return A(r.prepare(peer, idx)); }, py::arg("peer") = -1,
           py::arg("remote_buf_index") = 0)
      .def("build_context", [](Runtime& r) { return A(r.build_context()); })
      .def("reset", &Runtime::reset)
      .def("barrier", &Runtime::barrier, py::call_guard<py::gil_scoped_release>())
      .def_property_readonly("rank", &Runtime::rank)
      .def_property_readonly("size", &Runtime::size)
      .def_property_readonly("gpu_id", &Runtime::gpu_id)
      .def("clock_rate_khz", &Runtime::clock_rate_khz)
      .def("gpu_name", [](Runtime& r) { return std::string(r.gpu_name()); })
      .def("boot", &Runtime::boot_ptr)
      .def("put_no_db",
           [](Runtime& r, int src_idx, int dest_rank, int dest_idx, size_t size, size_t src_off, size_t dst_off) {
             Token t = r.put_no_db(to_buf(r, src_idx), dest_rank, dest_idx, size, src_off, dst_off);
             return py::make_tuple(t.slot, t.epoch);
           },
           py::arg("src_index"), py::arg("dest_rank"), py::arg("dest_index"), py::arg("size"), py::arg("src_off") = 0,
           py::arg("dst_off") = 0)
      .def("prepare_trigger", [](Runtime& r, int slot, uint64_t epoch) { return A(r.prepare_trigger(Token{slot, epoch})); })
      .def("wait", [](Runtime& r, int slot, uint64_t epoch) { r.wait(Token{slot, epoch}); },
           py::call_guard<py::gil_scoped_release>())
      .def("host_put",
           [](Runtime& r, uint64_t src, int dest_rank, int dest_buf, size_t dst_off, size_t size) {
             r.host_put(P<const void>(src), dest_rank, dest_buf, dst_off, size, cur_stream());
           })
      .def("host_get",
           [](Runtime& r, uint64_t dst, int src_rank, int src_buf, size_t src_off, size_t size) {
             r.host_get(P<void>(dst), src_rank, src_buf, src_off, size, cur_stream());
           })
      .def("signal_alloc", &Runtime::signal_alloc)
      .def("signal_local", [](Runtime& r, size_t w) { return A(r.signal_local(w)); }, py::arg("word") = 0)
      .def("signal_peer", [](Runtime& r, int rank, size_t w) { return A(r.signal_peer(rank, w)); }, py::arg("rank"),
           py::arg("word") = 0)
      .def("signal_multicast", [](Runtime& r, size_t w) { return A(r.signal_multicast(w)); }, py::arg("word") = 0)
      .def_property_readonly("timeout_ns", &Runtime::timeout_ns)
      .def("check_device_errors", &Runtime::check_device_errors, py::arg("clear") = true)
      .def("finalize", &Runtime::finalize, py::call_guard<py::gil_scoped_release>());

  py::class_<Barrier, std::shared_ptr<Barrier>>(m, "Barrier")
      .def(py::init<Runtime&, bool>(), py::arg("runtime"), py::arg("nvls") = false, py::keep_alive<1, 2>())
      .def("init", &Barrier::init)
      .def("finalize", &Barrier::finalize)
      .def("setup", &Barrier::setup)
      .def("wait_completion", &Barrier::wait_completion, py::call_guard<py::gil_scoped_release>())
      .def("reset", &Barrier::reset)
      .def("start_continuous", &Barrier::start_continuous)
      .def("wait_continuous", &Barrier::wait_continuous, py::call_guard<py::gil_scoped_release>())
      .def("device_ctx", [](Barrier& b) { return A(b.device_ctx()); })
      .def("advance", &Barrier::advance)
      .def("count", &Barrier::count)
      .def("inject_fault", &Barrier::inject_fault, py::arg("mode"), py::arg("epoch"), py::arg("timeout_ms") = 0)
      .def_property_readonly("next_epoch", &Barrier::next_epoch)
      .def_property_readonly("uses_nvls", &Barrier::uses_nvls);

  py::class_<CmdRing, std::shared_ptr<CmdRing>>(m, "CmdRing")
      .def(py::init<Runtime&, int, int, uint64_t>(), py::arg("runtime"), py::arg("nslots") = 64,
           py::arg("threads") = 256, py::arg("idle_timeout_ms") = 10000, py::keep_alive<1, 2>())
      .def("start", &CmdRing::start)
      .def("put", [](CmdRing& c, uint64_t src, int rank, int buf, size_t off, size_t size, uint64_t user) {
             return c.put(P<const void>(src), rank, buf, off, size, user);
           }, py::arg("src"), py::arg("dst_rank"), py::arg("dst_buf"), py::arg("dst_off"), py::arg("size"),
           py::arg("user") = 0)
      .def("get", [](CmdRing& c, uint64_t dst, int rank, int buf, size_t off, size_t size, uint64_t user) {
             return c.get(P<void>(dst), rank, buf, off, size, user);
           }, py::arg("dst"), py::arg("src_rank"), py::arg("src_buf"), py::arg("src_off"), py::arg("size"),
           py::arg("user") = 0)
      .def("signal", &CmdRing::signal, py::arg("dst_rank"), py::arg("word"), py::arg("value"))
      .def("add", &CmdRing::add, py::arg("dst_rank"), py::arg("word"), py::arg("value"))
      .def("fence", &CmdRing::fence)
      .def("wait", &CmdRing::wait, py::call_guard<py::gil_scoped_release>())
      .def("completed", &CmdRing::completed)
      .def("stop", &CmdRing::stop, py::call_guard<py::gil_scoped_release>())
      .def("status", &CmdRing::status)
      .def_property_readonly("running", &CmdRing::running);

  py::class_<am::Am, std::shared_ptr<am::Am>>(m, "Am")
      .def(py::init<Runtime&, int, uint32_t>(), py::arg("runtime"), py::arg("nslots") = am::AM_DEFAULT_RING_SLOTS,
           py::arg("max_payload") = am::AM_MAX_PAYLOAD_SIZE, py::keep_alive<1, 2>())
      .def("device_view", [](am::Am& a) { return A(a.device_view()); })
      .def_property_readonly("nslots", &am::Am::nslots)
      .def("send_handle",
           [](am::Am& a, int dst, int handler, std::vector<uint64_t> args, bool request) {
             am::am_args_t v{};
             for (size_t i = 0; i < args.size() && i < 6; ++i) v.data[i] = args[i];
             return a.send_handle(dst, (uint16_t)handler, v, request);
           },
           py::arg("dst"), py::arg("handler"), py::arg("args"), py::arg("request") = false)
      .def("send_payload",
           [](am::Am& a, int dst, int handler, std::vector<uint64_t> args, py::bytes payload) {
             am::am_args_t v{};
             for (size_t i = 0; i < args.size() && i < 6; ++i) v.data[i] = args[i];
             std::string p = payload;
             return a.send_payload(dst, (uint16_t)handler, v, p.data(), (uint32_t)p.size());
           })
      .def("check_can_send", &am::Am::check_can_send)
      .def("poll_once", &am::Am::poll_once, py::arg("max_per_peer") = 64)
      .def("reply", &am::Am::reply)
      .def("wait_reply", &am::Am::wait_reply, py::call_guard<py::gil_scoped_release>())
      .def("trigger_and_wait", &am::Am::trigger_and_wait)
      .def("counter", &am::Am::counter)
      .def("checksum", &am::Am::checksum);
  m.def("k_am_pingpong", [](uint64_t view, int peer, int iters, int mode, bool initiator, uint64_t out_ns) {
    ops::am_pingpong(P<am::AmView>(view), peer, iters, mode, initiator, P<unsigned long long>(out_ns), cur_stream());
  });

  // ---- communication kernels (enqueued on torch's current stream) ----
  m.def("k_barrier_single", [](uint64_t ctx, uint64_t flag) { ops::barrier_single(P<BarrierCtx>(ctx), P<uint64_t>(flag), cur_stream()); });
  m.def("k_barrier_continuous", [](uint64_t ctx, int n, uint64_t counter) {
    ops::barrier_continuous(P<BarrierCtx>(ctx), n, P<uint64_t>(counter), cur_stream());
  });
  m.def("k_copy", [](uint64_t dst, uint64_t src, size_t bytes, int iters, int blocks, int threads, size_t window) {
    ops::copy(P<void>(dst), P<const void>(src), bytes, iters, blocks, threads, cur_stream(), window);
  }, py::arg("dst"), py::arg("src"), py::arg("bytes"), py::arg("iters") = 1, py::arg("blocks") = 0, py::arg("threads") = 0,
     py::arg("window") = 0);
  m.def("k_put_signal", [](uint64_t dst, uint64_t src, size_t bytes, uint64_t sig, int blocks) {
    ops::put_signal(P<void>(dst), P<const void>(src), bytes, P<uint64_t>(sig), blocks, cur_stream());
  }, py::arg("dst"), py::arg("src"), py::arg("bytes"), py::arg("sig"), py::arg("blocks") = 0);
  m.def("k_wait_signal", [](uint64_t sig, int cmp, uint64_t value, uint64_t timeout_ns, uint64_t status) {
    ops::wait_signal(P<const uint64_t>(sig), cmp, value, timeout_ns, P<int>(status), cur_stream());
  });
  m.def("k_signal", [](uint64_t sig, uint64_t value, int op) { ops::signal(P<uint64_t>(sig), value, op, cur_stream()); });
  m.def("k_pingpong", [](uint64_t rbuf, uint64_t lbuf, size_t bytes, uint64_t rflag, uint64_t lflag, int iters,
                         bool initiator, uint64_t base, uint64_t out_ns, uint64_t timeout_ns, int rank) {
    ops::pingpong(P<void>(rbuf), P<const void>(lbuf), bytes, P<uint64_t>(rflag), P<const uint64_t>(lflag), iters,
                  initiator, base, P<uint64_t>(out_ns), timeout_ns, rank, cur_stream());
  });
  m.def("k_quiet_latency", [](uint64_t remote, int iters, uint64_t out_ns) {
    ops::quiet_latency(P<uint64_t>(remote), iters, P<uint64_t>(out_ns), cur_stream());
  });
  m.def("k_ctx_put", [](uint64_t ctx, uint64_t laddr, uint32_t lkey, uint64_t raddr, uint32_t rkey, uint32_t size) {
    ops::ctx_put(P<DeviceCtx>(ctx), laddr, lkey, raddr, rkey, size, cur_stream());
  });
  m.def("k_flush",[](uint64_t ctx, uint64_t status) { ops::flush_queued(P<DeviceCtx>(ctx), P<int>(status), cur_stream()); });
  m.def("k_reduce_bf16", [](std::vector<uint64_t> srcs, uint64_t out, size_t count, float scale, bool out_f32) {
    std::vector<const void*> p;
    for (auto a : srcs) p.push_back(P<const void>(a));
    ops::reduce_bf16(p.data(), (int)p.size(), P<void>(out), count, scale, out_f32, cur_stream());
  });
  m.def("k_allreduce_bf16", [](int algo, std::vector<uint64_t> in, std::vector<uint64_t> out, uint64_t mc_in,
                               uint64_t mc_out, int n, int me, size_t count, float scale, bool out_f32,
                               std::vector<uint64_t> flags, int max_blocks, uint64_t epoch, uint64_t timeout_ns,
                               int blocks, uint64_t epoch_dev, uint64_t ticket) {
    std::vector<const void*> ip;
    std::vector<void*> op;
    std::vector<uint64_t*> fp;
    for (auto a : in) ip.push_back(P<const void>(a));
    for (auto a : out) op.push_back(P<void>(a));
    for (auto a : flags) fp.push_back(P<uint64_t>(a));
    ops::allreduce_bf16(algo, ip.empty() ? nullptr : ip.data(), op.empty() ? nullptr : op.data(), P<const void>(mc_in),
                        P<void>(mc_out), n, me, count, scale, out_f32, fp.data(), max_blocks, epoch, timeout_ns, blocks,
                        cur_stream(), P<uint64_t>(epoch_dev), P<unsigned int>(ticket));
  }, py::arg("algo"), py::arg("in_ptrs"), py::arg("out_ptrs"), py::arg("mc_in"), py::arg("mc_out"), py::arg("n"),
     py::arg("me"), py::arg("count"), py::arg("scale"), py::arg("out_f32"), py::arg("flags"), py::arg("max_blocks"),
     py::arg("epoch"), py::arg("timeout_ns"), py::arg("blocks"), py::arg("epoch_dev") = 0, py::arg("ticket") = 0);
  m.def("k_reduce_scatter_bf16", [](bool nvls, std::vector<uint64_t> in, uint64_t mc_in, uint64_t out, int n, int me,
                                    size_t count, float scale, bool out_f32, std::vector<uint64_t> flags,
                                    int max_blocks, uint64_t epoch, uint64_t timeout_ns, int blocks, uint64_t epoch_dev,
                                    uint64_t ticket) {
    std::vector<const void*> ip;
    std::vector<uint64_t*> fp;
    for (auto a : in) ip.push_back(P<const void>(a));
    for (auto a : flags) fp.push_back(P<uint64_t>(a));
    if ((int)fp.size() != n || (!nvls && (int)ip.size() != n))
      throw std::runtime_error("k_reduce_scatter_bf16: one flag base (and, without NVLS, one input) per rank");
    ops::reduce_scatter_bf16(nvls, ip.empty() ? nullptr : ip.data(), P<const void>(mc_in), P<void>(out), n, me, count,
                             scale, out_f32, fp.data(), max_blocks, epoch, timeout_ns, blocks, cur_stream(),
                             P<uint64_t>(epoch_dev), P<unsigned int>(ticket));
  }, py::arg("nvls"), py::arg("in_ptrs"), py::arg("mc_in"), py::arg("out"), py::arg("n"), py::arg("me"),
     py::arg("count"), py::arg("scale"), py::arg("out_f32"), py::arg("flags"), py::arg("max_blocks"), py::arg("epoch"),
     py::arg("timeout_ns"), py::arg("blocks") = 0, py::arg("epoch_dev") = 0, py::arg("ticket") = 0);
  m.def("k_all_gather", [](bool nvls, uint64_t shard, std::vector<uint64_t> out, uint64_t mc_out, int n, int me,
                           size_t shard_bytes, std::vector<uint64_t> flags, int max_blocks, uint64_t epoch,
                           uint64_t timeout_ns, int blocks, uint64_t epoch_dev, uint64_t ticket) {
    std::vector<void*> op;
    std::vector<uint64_t*> fp;
    for (auto a : out) op.push_back(P<void>(a));
    for (auto a : flags) fp.push_back(P<uint64_t>(a));
    if ((int)fp.size() != n || (!nvls && (int)op.size() != n))
      throw std::runtime_error("k_all_gather: one flag base (and, without NVLS, one output) per rank");
    ops::all_gather(nvls, P<const void>(shard), op.empty() ? nullptr : op.data(), P<void>(mc_out), n, me, shard_bytes,
                    fp.data(), max_blocks, epoch, timeout_ns, blocks, cur_stream(), P<uint64_t>(epoch_dev),
                    P<unsigned int>(ticket));
  }, py::arg("nvls"), py::arg("shard"), py::arg("out_ptrs"), py::arg("mc_out"), py::arg("n"), py::arg("me"),
     py::arg("shard_bytes"), py::arg("flags"), py::arg("max_blocks"), py::arg("epoch"), py::arg("timeout_ns"),
     py::arg("blocks") = 0, py::arg("epoch_dev") = 0, py::arg("ticket") = 0);
  m.def("k_jacobi_init", [](uint64_t a, uint64_t b, int nx, int ny, int rows, int g0, uint64_t seed) {
    ops::jacobi_init(P<float>(a), P<float>(b), nx, ny, rows, g0, seed, cur_stream());
  });
  m.def("jacobi_persistent_grid", &ops::jacobi_persistent_grid, py::arg("rows"));
  m.def("k_jacobi_run", [](py::dict d) {
    ops::JacobiRun r;
    auto u64 = [&](const char* k) { return d.contains(k) ? d[k].cast<uint64_t>() : (uint64_t)0; };
    auto two = [&](const char* k, int i) {
      return d.contains(k) ? d[k].cast<std::vector<uint64_t>>().at(i) : (uint64_t)0;
    };
    for (int i = 0; i < 2; ++i) {
      r.buf[i] = P<float>(two("buf", i));
      r.top_dst[i] = P<float>(two("top_dst", i));
      r.bot_dst[i] = P<float>(two("bot_dst", i));
    }
    r.nx = d["nx"].cast<int>();
    r.rows = d["rows"].cast<int>();
    r.top_sig_remote = P<uint64_t>(u64("top_sig_remote"));
    r.bot_sig_remote = P<uint64_t>(u64("bot_sig_remote"));
    r.top_flag = P<const uint64_t>(u64("top_flag"));
    r.bot_flag = P<const uint64_t>(u64("bot_flag"));
    r.iter0 = u64("iter0");
    r.iters = d["iters"].cast<int>();
    r.done = P<uint64_t>(u64("done"));
    r.norm = P<double>(u64("norm"));
    r.timeout_ns = u64("timeout_ns");
    r.rank = d.contains("rank") ? d["rank"].cast<int>() : 0;
    ops::jacobi_run(r, cur_stream());
  });
  m.def("k_jacobi_step", [](uint64_t a, uint64_t b, int nx, int rows, uint64_t top_dst, uint64_t bot_dst,
                            uint64_t top_sig_remote, uint64_t bot_sig_remote, uint64_t top_flag, uint64_t bot_flag,
                            uint64_t wait_top, uint64_t wait_bot, uint64_t norm, uint64_t timeout_ns, int rank) {
    ops::JacobiStep st;
    st.a = P<const float>(a);
    st.b = P<float>(b);
    st.nx = nx;
    st.rows = rows;
    st.top_dst = P<float>(top_dst);
    st.bot_dst = P<float>(bot_dst);
    st.top_sig_remote = P<uint64_t>(top_sig_remote);
    st.bot_sig_remote = P<uint64_t>(bot_sig_remote);
    st.top_flag = P<const uint64_t>(top_flag);
    st.bot_flag = P<const uint64_t>(bot_flag);
    st.wait_top = wait_top;
    st.wait_bot = wait_bot;
    st.norm = P<double>(norm);
    st.timeout_ns = timeout_ns;
    st.rank = rank;
    ops::jacobi_step(st, cur_stream());
  });
  m.def("jacobi_ctas_per_row", &ops::jacobi_ctas_per_row);
  m.def("k_ag_gemm", [](int n, int r, int M, int Ns, int K, std::vector<uint64_t> a_full, uint64_t B, long long ldb,
                        uint64_t C, long long ldc, std::vector<uint64_t> arrivals, std::vector<uint64_t> done,
                        uint64_t epoch, int units_per_band, int grid, uint64_t timeout_ns, uint64_t trace,
                        int diag, int comm_ctas, uint64_t tile_counter, uint64_t a_mc, uint64_t arrivals_mc,
                        int pair) {
    if ((int)a_full.size() != n || (int)arrivals.size() != n || (int)done.size() != n || n > 16)
      throw std::runtime_error("k_ag_gemm: per-rank pointer lists must have n <= 16 entries");
    ops::AgGemmArgs a;
    a.n = n; a.r = r; a.M = M; a.Ns = Ns; a.K = K;
    for (int i = 0; i < n; ++i) {
      a.a_full[i] = P<void>(a_full[i]);
      a.arrivals[i] = P<uint64_t>(arrivals[i]);
      a.done[i] = P<uint64_t>(done[i]);
    }
    a.B = P<const void>(B); a.ldb = ldb; a.C = P<void>(C); a.ldc = ldc;
    a.epoch = epoch; a.units_per_band = units_per_band; a.grid = grid; a.timeout_ns = timeout_ns;
    a.trace = P<uint64_t>(trace); a.diag = diag; a.comm_ctas = comm_ctas;
    a.tile_counter = P<uint64_t>(tile_counter);
    a.a_mc = P<void>(a_mc); a.arrivals_mc = P<uint64_t>(arrivals_mc);
    a.pair = pair;
    ops::ag_gemm(a, cur_stream());
  }, py::arg("n"), py::arg("r"), py::arg("M"), py::arg("Ns"), py::arg("K"), py::arg("a_full"), py::arg("B"),
     py::arg("ldb"), py::arg("C"), py::arg("ldc"), py::arg("arrivals"), py::arg("done"), py::arg("epoch"),
     py::arg("units_per_band"), py::arg("grid"), py::arg("timeout_ns"), py::arg("trace") = 0, py::arg("diag") = 0,
     py::arg("comm_ctas") = 0, py::arg("tile_counter") = 0, py::arg("a_mc") = 0, py::arg("arrivals_mc") = 0,
     py::arg("pair") = 0);
  m.def("ag_transfer_ce", [](int n, int r, int M, int K, std::vector<uint64_t> a_full, std::vector<uint64_t> arrivals,
                             uint64_t done_local, uint64_t epoch, int grid, int units_per_band, int chunks,
                             uint64_t timeout_ns) {
    if ((int)a_full.size() != n || (int)arrivals.size() != n || n > 16)
      throw std::runtime_error("ag_transfer_ce: per-rank pointer lists must have n <= 16 entries");
    ops::AgCeArgs a;
    a.n = n; a.r = r; a.M = M; a.K = K;
    for (int i = 0; i < n; ++i) {
      a.a_full[i] = P<void>(a_full[i]);
      a.arrivals[i] = P<uint64_t>(arrivals[i]);
    }
    a.done_local = P<const uint64_t>(done_local);
    a.epoch = epoch; a.grid = grid; a.units_per_band = units_per_band; a.chunks = chunks;
    a.timeout_ns = timeout_ns;
    ops::ag_transfer_ce(a, cur_stream());
  }, py::arg("n"), py::arg("r"), py::arg("M"), py::arg("K"), py::arg("a_full"), py::arg("arrivals"),
     py::arg("done_local"), py::arg("epoch"), py::arg("grid"), py::arg("units_per_band"), py::arg("chunks"),
     py::arg("timeout_ns") = 0);
  m.def("k_gemm_rs", [](int n, int r, int M, int N, int K, uint64_t A, long long lda, uint64_t B, long long ldb,
                        std::vector<uint64_t> slots, std::vector<uint64_t> arrivals, std::vector<uint64_t> done,
                        uint64_t out, long long ldo, uint64_t epoch, int grid, uint64_t timeout_ns,
                        uint64_t staging_mc, uint64_t band_tiles, uint64_t tile_counter, int comm_ctas,
                        int units_per_band, uint64_t trace, int join_reduce, uint64_t unit_counter,
                        int raster_group, int pair) {
    if ((int)slots.size() != n || (int)arrivals.size() != n || (int)done.size() != n || n > 16)
      throw std::runtime_error("k_gemm_rs: per-rank pointer lists must have n <= 16 entries");
    ops::GemmRsArgs a;
    a.n = n; a.r = r; a.M = M; a.N = N; a.K = K;
    a.A = P<const void>(A); a.lda = lda; a.B = P<const void>(B); a.ldb = ldb;
    for (int i = 0; i < n; ++i) {
      a.slots[i] = P<void>(slots[i]);
      a.arrivals[i] = P<uint64_t>(arrivals[i]);
      a.done[i] = P<uint64_t>(done[i]);
    }
    a.out = P<void>(out); a.ldo = ldo; a.epoch = epoch; a.grid = grid; a.timeout_ns = timeout_ns;
    a.staging_mc = P<const void>(staging_mc); a.band_tiles = P<uint64_t>(band_tiles);
    a.tile_counter = P<uint64_t>(tile_counter); a.comm_ctas = comm_ctas; a.units_per_band = units_per_band;
    a.trace = P<uint64_t>(trace);
    a.join_reduce = join_reduce; a.unit_counter = P<uint64_t>(unit_counter);
    a.raster_group = raster_group;
    a.pair = pair;
    ops::gemm_rs(a, cur_stream());
  }, py::arg("n"), py::arg("r"), py::arg("M"), py::arg("N"), py::arg("K"), py::arg("A"), py::arg("lda"), py::arg("B"),
     py::arg("ldb"), py::arg("slots"), py::arg("arrivals"), py::arg("done"), py::arg("out"), py::arg("ldo"),
     py::arg("epoch"), py::arg("grid"), py::arg("timeout_ns"), py::arg("staging_mc") = 0, py::arg("band_tiles") = 0,
     py::arg("tile_counter") = 0, py::arg("comm_ctas") = 0, py::arg("units_per_band") = 4, py::arg("trace") = 0,
     py::arg("join_reduce") = 0, py::arg("unit_counter") = 0, py::arg("raster_group") = 0, py::arg("pair") = 0);
  m.def("k_litmus", [](int test, int iters, int k, int use_fence, uint32_t seed, uint32_t max_delay, uint64_t timeout_ns,
                       int role_base, int nroles_here, std::vector<std::vector<uint64_t>> roles) {
    if (roles.size() != 2) throw std::runtime_error("k_litmus: two role pointer lists");
    ops::LitmusArgs a;
    a.test = test; a.iters = iters; a.k = k; a.use_fence = use_fence; a.seed = seed; a.max_delay = max_delay;
    a.timeout_ns = timeout_ns; a.role_base = role_base;
    for (int r = 0; r < 2; ++r) {
      const auto& v = roles[r];
      if (v.size() != 8) throw std::runtime_error("k_litmus: 8 pointers per role");
      a.role[r].data = P<uint64_t>(v[0]); a.role[r].flag = P<uint64_t>(v[1]);
      a.role[r].ready_remote = P<uint64_t>(v[2]); a.role[r].ready_local = P<const uint64_t>(v[3]);
      a.role[r].mine_remote = P<uint64_t>(v[4]); a.role[r].theirs_local = P<const uint64_t>(v[5]);
      a.role[r].out = P<uint64_t>(v[6]); a.role[r].result = P<uint64_t>(v[7]);
    }
    ops::litmus(a, nroles_here, cur_stream());
  }, py::arg("test"), py::arg("iters"), py::arg("k"), py::arg("use_fence"), py::arg("seed"), py::arg("max_delay"),
     py::arg("timeout_ns"), py::arg("role_base"), py::arg("nroles_here"), py::arg("roles"));
  m.def("k_phase_loop", [](uint64_t bar, uint64_t x, uint64_t y, uint64_t recv, uint64_t send_remote, size_t n,
                           int iters, float a, int rank, int left, uint64_t stamps, uint64_t bad) {
    ops::phase_loop(P<BarrierCtx>(bar), P<float>(x), P<float>(y), P<const float>(recv), P<float>(send_remote), n, iters,
                    a, rank, left, P<uint64_t>(stamps), P<unsigned long long>(bad), cur_stream());
  });
  m.def("k_saxpy_put", [](uint64_t x, uint64_t y, float a, size_t n, uint64_t dst_remote, uint64_t arrivals_remote,
                          int blocks) {
    ops::saxpy_put(P<const float>(x), P<float>(y), a, n, P<float>(dst_remote), P<uint64_t>(arrivals_remote), blocks,
                   cur_stream());
  });
  m.def("k_wait_count", [](uint64_t counter, uint64_t target, uint64_t timeout_ns, int rank) {
    ops::wait_count(P<const uint64_t>(counter), target, timeout_ns, rank, cur_stream());
  });
  m.def("ring_mm_grid", &ops::ring_mm_grid, py::arg("Ns"), py::arg("push_ctas"));
  m.def("ring_mm_grid_tc", &ops::ring_mm_grid_tc, py::arg("push_ctas"));
  m.def("tf32_split", [](uint64_t src, long long ld, int rows, int K, uint64_t dst, int order) {
    ops::tf32_split(P<const float>(src), ld, rows, K, P<float>(dst), order, cur_stream());
  }, py::arg("src"), py::arg("ld"), py::arg("rows"), py::arg("K"), py::arg("dst"), py::arg("order"));
  m.def("k_ring_mm_step", [](py::dict d) {
    ops::RingMmStep a;
    auto u64 = [&](const char* k) { return d.contains(k) ? d[k].cast<uint64_t>() : (uint64_t)0; };
    a.N = d["N"].cast<int>();
    a.Ns = d["Ns"].cast<int>();
    a.A = P<const float>(u64("A"));
    a.Bcur = P<const float>(u64("Bcur"));
    a.C = P<float>(u64("C"));
    a.col_block = d["col_block"].cast<int>();
    a.Bnext_remote = P<float>(u64("Bnext_remote"));
    a.arrivals_remote = P<uint64_t>(u64("arrivals_remote"));
    a.arrivals = P<const uint64_t>(u64("arrivals"));
    a.arrivals_target = u64("arrivals_target");
    a.consumed = P<const uint64_t>(u64("consumed"));
    a.consumed_target = u64("consumed_target");
    a.consumed_left = P<uint64_t>(u64("consumed_left"));
    a.ticket = P<unsigned long long>(u64("ticket"));
    a.ticket_target = u64("ticket_target");
    a.push_ctas = d.contains("push_ctas") ? d["push_ctas"].cast<int>() : 0;
    a.timeout_ns = u64("timeout_ns");
    a.rank = d.contains("rank") ? d["rank"].cast<int>() : 0;
    a.left = d.contains("left") ? d["left"].cast<int>() : -1;
    a.right = d.contains("right") ? d["right"].cast<int>() : -1;
    a.Asplit = P<const float>(u64("Asplit"));
    a.Bsplit = P<float>(u64("Bsplit"));
    ops::ring_mm_step(a, cur_stream());
  });
  m.def("k_put_tile", [](uint64_t dst, int tiles, uint32_t tile_bytes, uint32_t seed, uint64_t sig) {
    ops::put_tile_test(P<void>(dst), tiles, tile_bytes, seed, P<uint64_t>(sig), cur_stream());
  }, py::arg("dst"), py::arg("tiles"), py::arg("tile_bytes"), py::arg("seed"), py::arg("sig") = 0);
  m.def("k_saxpy", [](uint64_t x, uint64_t y, float a, size_t n) {
    ops::saxpy(P<const float>(x), P<float>(y), a, n, cur_stream());
  });
  m.def("k_moe_route", [](uint64_t logits, int T, int E, int topk, uint64_t idx, uint64_t w, uint64_t counts) {
    ops::moe_route(P<const float>(logits), T, E, topk, P<int>(idx), P<float>(w), P<int>(counts), cur_stream());
  });
  m.def("k_moe_forward", [](py::dict d) {
    ops::MoeArgs a;
    a.n = d["n"].cast<int>();
    a.r = d["r"].cast<int>();
    a.T = d["T"].cast<int>();
    a.H = d["H"].cast<int>();
    a.I = d["I"].cast<int>();
    a.E = d["E"].cast<int>();
    a.topk = d["topk"].cast<int>();
    a.logits = P<const float>(d["logits"].cast<uint64_t>());
    a.x = P<const void>(d["x"].cast<uint64_t>());
    a.w1 = P<const void>(d["w1"].cast<uint64_t>());
    a.w2 = P<const void>(d["w2"].cast<uint64_t>());
    a.topk_idx = P<int>(d["topk_idx"].cast<uint64_t>());
    a.topk_w = P<float>(d["topk_w"].cast<uint64_t>());
    a.counts = P<int>(d["counts"].cast<uint64_t>());
    auto vec = [&](const char* k) { return d[k].cast<std::vector<uint64_t>>(); };
    auto ct = vec("count_tab"), pf = vec("plan_flags"), rv = vec("recv"), mt = vec("meta"), ar = vec("arrivals"),
         cb = vec("comb"), ca = vec("comb_arrivals");
    if ((int)ct.size() != a.n || a.n > 8) throw std::runtime_error("k_moe_forward: per-rank lists need n <= 8 entries");
    for (int i = 0; i < a.n; ++i) {
      a.count_tab[i] = P<void>(ct[i]);
      a.plan_flags[i] = P<uint64_t>(pf[i]);
      a.recv[i] = P<void>(rv[i]);
      a.meta[i] = P<void>(mt[i]);
      a.arrivals[i] = P<uint64_t>(ar[i]);
      a.comb[i] = P<void>(cb[i]);
      a.comb_arrivals[i] = P<uint64_t>(ca[i]);
    }
    a.h = P<void>(d["h"].cast<uint64_t>());
    a.out = P<void>(d["out"].cast<uint64_t>());
    a.cap_rows = d["cap_rows"].cast<int>();
    a.epoch = d["epoch"].cast<uint64_t>();
    a.timeout_ns = d["timeout_ns"].cast<uint64_t>();
    py::dict w = d["ws"];
    a.ws.dest_row_base = P<int>(w["dest_row_base"].cast<uint64_t>());
    a.ws.key_base = P<int>(w["key_base"].cast<uint64_t>());
    a.ws.key_cursor = P<int>(w["key_cursor"].cast<uint64_t>());
    a.ws.expert_base = P<int>(w["expert_base"].cast<uint64_t>());
    a.ws.expert_rows = P<int>(w["expert_rows"].cast<uint64_t>());
    a.ws.mblk_prefix = P<int>(w["mblk_prefix"].cast<uint64_t>());
    a.ws.cum_rows = P<uint64_t>(w["cum_rows"].cast<uint64_t>());
    a.ws.cum_pairs = P<uint64_t>(w["cum_pairs"].cast<uint64_t>());
    a.ws.send_pair = P<int>(w["send_pair"].cast<uint64_t>());
    a.ws.send_row = P<int>(w["send_row"].cast<uint64_t>());
    if (w.contains("g1_tile_ctr")) a.ws.g1_tile_ctr = P<uint64_t>(w["g1_tile_ctr"].cast<uint64_t>());
    if (w.contains("g2_ctr")) a.ws.g2_ctr = P<uint64_t>(w["g2_ctr"].cast<uint64_t>());
    if (w.contains("g2_queue")) a.ws.g2_queue = P<uint64_t>(w["g2_queue"].cast<uint64_t>());
    if (d.contains("dispatch_ctas")) a.dispatch_ctas = d["dispatch_ctas"].cast<int>();
    if (d.contains("combine_ctas")) a.combine_ctas = d["combine_ctas"].cast<int>();
    if (d.contains("comm_only")) a.comm_only = d["comm_only"].cast<int>();
    if (d.contains("y_stage")) a.y_stage = P<void>(d["y_stage"].cast<uint64_t>());
    std::vector<float> stage(6, 0.f);
    const bool timed = d.contains("stage_times") && d["stage_times"].cast<bool>();
    if (timed) a.stage_ms = stage.data();
    ops::moe_forward(a, cur_stream());
    py::list out;
    if (timed)
      for (float v : stage) out.append(v);
    return out;
  });
  m.def("k_fill_pattern", [](uint64_t buf, size_t n, uint32_t seed) { ops::fill_pattern(P<void>(buf), n, seed, cur_stream()); });
  m.def("k_check_pattern_range", [](uint64_t buf, size_t n, uint32_t seed, size_t base, uint64_t bad) {
    ops::check_pattern(P<const void>(buf), n, seed, P<unsigned long long>(bad), cur_stream(), base);
  });
  m.def("k_check_pattern", [](uint64_t buf, size_t n, uint32_t seed, uint64_t bad) {
    ops::check_pattern(P<const void>(buf), n, seed, P<unsigned long long>(bad), cur_stream());
  });
}
