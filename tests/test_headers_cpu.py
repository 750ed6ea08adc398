"""The umbrella headers under the reference's names compile: <gicc/gicc.hpp> with the host
compiler and <gicc/gicc_device.cuh> in an sm_100a translation unit, so a program written for
the reference finds its includes."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INC = os.path.join(ROOT, "csrc", "include")
NVCC = "/usr/local/cuda/bin/nvcc"


def test_host_umbrella_header(tmp_path):
    if shutil.which("g++") is None:
        pytest.skip("no g++")
    src = tmp_path / "h.cpp"
    src.write_text("#include <gicc/gicc.hpp>\n#include <gicc/bootstrap/bootstrap.hpp>\n#include <gicc/coll.hpp>\n"
                   "int main() { return gicc::config().timeout_ms == 0; }\n")
    p = subprocess.run(["g++", "-std=c++17", f"-I{INC}", "-I/usr/local/cuda/include", "-fsyntax-only", str(src)],
                       capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stderr[-3000:]


def test_device_umbrella_header(tmp_path):
    if not os.path.exists(NVCC):
        pytest.skip("no nvcc")
    src = tmp_path / "d.cu"
    src.write_text("#include <gicc/gicc.hpp>\n#include <gicc/gicc_device.cuh>\n"
                   "__global__ void k(gicc::DeviceCtx* c, uint64_t l, uint32_t lk, uint64_t r, uint32_t rk) {\n"
                   "  gicc::put(c, l, lk, r, rk, 64);\n  gicc::flush(c);\n  gicc::quiet(c);\n}\n")
    p = subprocess.run([NVCC, "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", f"-I{INC}",
                        "--expt-relaxed-constexpr", "-c", str(src), "-o", str(tmp_path / "d.o")],
                       capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-3000:]


def test_reference_style_program_compiles(tmp_path):
    """A program written against the reference's documented API (Runtime register_buffer /
    exchange / prepare / remote_buffer / reset, device put / flush / quiet on a DeviceCtx,
    Barrier continuous mode) compiles unchanged against these headers."""
    if not os.path.exists(NVCC):
        pytest.skip("no nvcc")
    src = tmp_path / "app.cu"
    src.write_text(r"""
#include <gicc/gicc.hpp>
#include <gicc/gicc_device.cuh>
#include <gicc/gicc_types.hpp>
__global__ void simple(gicc::GiccContext* ctx, float* x, size_t n, int peer) {
  float* dst = static_cast<float*>(gicc::remote_ptr(ctx, x, peer));
  gicc::put(ctx, dst, x, (uint32_t)(n * sizeof(float)), peer);
  gicc::put_no_db(ctx, dst, x, (uint32_t)(n * sizeof(float)), peer);
  gicc::flush(ctx, peer);
  gicc::quiet(ctx, peer);
}
__global__ void kernel(gicc::DeviceCtx* ctx, uint64_t laddr, uint32_t lkey, uint64_t raddr, uint32_t rkey,
                       uint32_t size, gicc::BarrierCtx* bar) {
  gicc::put(ctx, laddr, lkey, raddr, rkey, size);
  gicc::quiet(ctx);
  gicc::flush(ctx);
  gicc::barrier(bar);
  bar->expected_signal++;
}
int main() {
  gicc::Runtime rt;
  void* d = nullptr;
  cudaMalloc(&d, 1 << 20);
  auto buf = rt.register_buffer(d, 1 << 20, true);
  rt.exchange();
  const int peer = (rt.rank() + 1) % rt.size();
  auto remote = rt.remote_buffer(peer, buf.index);
  gicc::DeviceCtx* ctx = rt.prepare(peer, buf.index);
  gicc::Barrier barrier(rt);
  barrier.setup();
  kernel<<<1, 32>>>(ctx, buf.addr, buf.lkey, remote.addr, remote.rkey, 4096, barrier.device_ctx());
  barrier.wait_completion();
  // OFI-style host queue: put_no_db -> Token, prepare_trigger, device flush, host wait
  gicc::Token t = rt.put_no_db(buf, peer, buf.index, 4096, 0, 0);
  gicc::DeviceCtx* tctx = rt.prepare_trigger(t);
  kernel<<<1, 32>>>(tctx, buf.addr, buf.lkey, remote.addr, remote.rkey, 0, barrier.device_ctx());
  rt.wait(t);
  // continuous barrier mode
  barrier.start_continuous(100);
  barrier.wait_continuous();
  // the OFI programs' spelling: a transport over a caller-owned bootstrap
  {
    gicc::Bootstrap boot;
    gicc::Fabric comm(boot);
    gicc::Barrier b2(comm.fabric());
    (void)comm.gpu_id();
  }
  // active messages
  gicc::am::Am am(rt);
  gicc::am::am_args_t args{};
  am.send_handle(peer, 1, args);
  am.poll_once();
  rt.barrier();
  rt.reset();
  // NVSHMEM-style simplified API
  gicc::init();
  float* x = static_cast<float*>(gicc::malloc(1 << 20));
  simple<<<1, 32>>>(gicc::context(), x, 1024, (gicc::my_pe() + 1) % gicc::n_pes());
  gicc::barrier();
  gicc::free(x);
  gicc::finalize();
  return 0;
}
""")
    p = subprocess.run([NVCC, "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", f"-I{INC}",
                        "--expt-relaxed-constexpr", "-c", str(src), "-o", str(tmp_path / "app.o")],
                       capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-3000:]


def test_c_api_headers_under_reference_names(tmp_path):
    """Programs include "gda.h" / "gda_barrier_proxy.h" with include/ and include/gda on the
    path (the CMake target exports both), as the reference's C API programs do."""
    if shutil.which("g++") is None:
        pytest.skip("no g++")
    src = tmp_path / "c.cpp"
    src.write_text('#include "gda.h"\n#include "gda_barrier_proxy.h"\nint main() { return gda_rank() < -1; }\n')
    p = subprocess.run(["g++", "-std=c++17", f"-I{INC}", f"-I{os.path.join(INC, 'gda')}", "-I/usr/local/cuda/include",
                        "-fsyntax-only", str(src)], capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stderr[-3000:]
