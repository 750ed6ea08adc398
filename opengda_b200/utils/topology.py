"""Node topology probe: what the GPUs of this node report about one another.

* ``p2p``: for every ordered pair of visible GPUs, cudaDeviceGetP2PAttribute's access,
  native-atomics, CUDA-array and performance-rank values (native ``p2p_links``);
* ``nvlink``: per GPU, how many NVLink links NVML reports active, and their version
  (read-only NVML queries; skipped when NVML is not importable);
* ``uniform``: True when every pair has access and native atomics with one performance rank
  -- what an NVSwitch node reports, and what the runtime's peer mappings and signal atomics
  assume.

The runtime needs none of this (every peer of an NVSwitch node is equivalent); it is a
sanity check to run on a new node.  ``python -m opengda_b200.utils.topology`` prints it as JSON.
The NVML module and the P2P query are parameters so the logic is testable without a GPU.
"""
from __future__ import annotations

import json
from typing import Any, Callable, Dict, List, Optional

NVLINK_MAX_LINKS = 18  # NVLink 5 on B200


def _nvlink_state(nvml) -> List[Dict[str, Any]]:
    out = []
    nvml.nvmlInit()
    try:
        for i in range(nvml.nvmlDeviceGetCount()):
            h = nvml.nvmlDeviceGetHandleByIndex(i)
            name = nvml.nvmlDeviceGetName(h)
            if isinstance(name, bytes):
                name = name.decode()
            active, versions = 0, set()
            for link in range(NVLINK_MAX_LINKS):
                try:
                    if nvml.nvmlDeviceGetNvLinkState(h, link):
                        active += 1
                        try:
                            versions.add(int(nvml.nvmlDeviceGetNvLinkVersion(h, link)))
                        except Exception:  # version query unsupported: keep the count
                            pass
                except Exception:  # link index not present on this part
                    break
            out.append({"index": i, "name": name, "active_links": active, "versions": sorted(versions)})
    finally:
        nvml.nvmlShutdown()
    return out


def probe(nvml: Any = "import", p2p: Optional[Callable[[], List[Dict[str, int]]]] = None) -> Dict[str, Any]:
    """The node's GPU peer matrix and NVLink state (see the module docstring)."""
    if p2p is None:
        from .. import native
        p2p = native().p2p_links
    links = list(p2p())
    res: Dict[str, Any] = {"p2p": links}
    if nvml == "import":
        try:
            import pynvml as nvml  # nvidia-ml-py
        except ImportError:
            nvml = None
    try:
        res["nvlink"] = _nvlink_state(nvml) if nvml is not None else None
    except Exception as e:  # NVML present but not usable here (driver or permissions)
        res["nvlink"] = None
        res["nvml_error"] = f"{type(e).__name__}: {e}"
    ranks = {l["perf_rank"] for l in links}
    res["uniform"] = bool(links) and all(l["access"] and l["native_atomics"] for l in links) and len(ranks) == 1
    missing = [(l["src"], l["dst"]) for l in links if not l["access"]]
    res["pairs_without_access"] = missing
    return res


def environment() -> Dict[str, Any]:
    """Versions of what this package runs on (the reference's scripts check their module
    environment the same way before a run): Python, torch and its CUDA / NCCL, the driver
    (NVML), nvcc, the visible GPUs and whether the native library loads."""
    import platform
    import shutil
    import subprocess

    env: Dict[str, Any] = {"python": platform.python_version()}
    try:
        import torch
        env["torch"] = torch.__version__
        env["torch_cuda"] = torch.version.cuda
        env["cuda_available"] = torch.cuda.is_available()
        if torch.cuda.is_available():
            env["gpus"] = [torch.cuda.get_device_name(i) for i in range(torch.cuda.device_count())]
            try:
                env["nccl"] = ".".join(map(str, torch.cuda.nccl.version()))
            except Exception as e:  # NCCL not bundled
                env["nccl"] = f"unavailable: {e}"
    except ImportError:
        env["torch"] = None
    try:
        import pynvml
        pynvml.nvmlInit()
        try:
            v = pynvml.nvmlSystemGetDriverVersion()
            env["driver"] = v.decode() if isinstance(v, bytes) else v
        finally:
            pynvml.nvmlShutdown()
    except Exception as e:
        env["driver"] = f"unavailable: {type(e).__name__}"
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    try:
        out = subprocess.run([nvcc, "--version"], capture_output=True, text=True, timeout=30).stdout
        env["nvcc"] = out.strip().splitlines()[-1] if out.strip() else None
    except (OSError, subprocess.SubprocessError):
        env["nvcc"] = None
    try:
        from .. import native
        native()
        env["native_library"] = "loaded"
    except Exception as e:
        env["native_library"] = f"not loadable: {e}"
    return env


def main() -> None:
    res: Dict[str, Any] = {"environment": environment()}
    try:
        res["topology"] = probe()
    except Exception as e:  # no GPU here
        res["topology"] = f"unavailable: {type(e).__name__}: {e}"
    print(json.dumps(res, indent=1))


if __name__ == "__main__":
    main()
