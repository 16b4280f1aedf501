"""Build and load the in-tree sm_100a extension (``pra_ops``).

``build()`` compiles every kernel translation unit for ``sm_100a`` with ninja
(incremental, parallel) into ``pdattention_b200/ops/_build/`` and imports the
result.  ``load()`` imports an already-built module without invoking the
compiler, so a machine that received the built ``.so`` never recompiles.
``require()`` is what the CUDA code paths call: it raises when the extension
is missing instead of silently falling back to a slower path.
"""

from __future__ import annotations

import importlib.machinery
import importlib.util
import os
import sys
import sysconfig
from pathlib import Path

NAME = "pra_ops"
ROOT = Path(__file__).resolve().parents[2]
CSRC = ROOT / "csrc"
BUILD_DIR = Path(__file__).resolve().parent / "_build"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]

_SOURCES = ["bindings.cpp", "attention.cu", "attention_tc.cu", "norm.cu", "loss_optim.cu", "gist.cu", "routing.cu", "llama.cu",
            "gemm/tn_bias.cu", "gemm/tn_bias_gelu.cu", "gemm/nn.cu", "gemm/nn_dgelu.cu", "gemm/wgrad.cu", "gemm/tn_f32.cu", "gemm/tn_bias_small.cu", "gemm/tn_bias_narrow.cu", "gemm/nn_sk.cu", "gemm/wgrad_sk.cu", "gemm/dispatch.cu",
            "planner.cpp", "decode_gemm.cu", "dropout.cu", "colsum_noalloc.cu", "dp_reduce.cu", "tp_comm.cu", "embed.cu", "driver_shim.cu"]

_module = None

# Kernels launched per extension call (used to report how many of this library's
# kernels ran inside a timed region).
KERNELS_PER_CALL = {"attention_fwd": 1, "attention_bwd": 3, "gemm": 1, "norm_fwd": 1, "norm_bwd": 3, "colsum": 2,
                    "cross_entropy": 1, "grad_norm": 2, "adamw": 1, "gist_mean": 1, "gist_kmeans": 1, "route": 1,
                    "gist_mean_into": 1, "gist_kmeans_into": 1,
                    "stack_forward": 0, "stack_train_forward": 0, "stack_train_backward": 0, "dp_allreduce": 1, "dp_signal_words": 0,
                    "ipc_alloc": 0, "ipc_open": 0, "ipc_close": 0,
                    "rope_copy": 1, "silu_mul": 1, "decode_prologue": 1, "decode_attention": 2, "route_topk": 1,
                    "tp_allreduce": 1, "tp_allgather": 1, "tp_signal_words": 0, "route_merge": 1, "embed_add": 1, "combine_partials": 1, "attention_status": 0, "plan_batch": 0, "decode_gemm": 1, "decode_qkv_rope": 1, "decode_gemm_max_tiles": 0, "decode_gemm_flag_slots": 0, "decode_gemm_resident_clusters": 0, "set_attention_impl": 0, "attention_impl": 0,
                    "dropout": 1, "dropout_add": 1, "decode_set_tma": 0, "set_pdl": 0, "pdl_enabled": 0, "gelu_probe": 1, "set_launch_priority": 0, "decode_set_stages": 0, "decode_gemm_configure": 0, "route_topk_exchange": 1, "set_bounds_check": 0, "bounds_check_enabled": 0, "bounds_status": 0, "bounds_reset": 0}  # stack_*: counted per layer by their callers


class LaunchCounter:
    """Proxy around the extension that counts kernel launches while enabled."""

    def __init__(self, module):
        self._module = module
        self.enabled = False
        self.launches = 0
        self.calls: dict[str, int] = {}

    def __getattr__(self, name):
        fn = getattr(self._module, name)
        if not callable(fn):
            return fn

        def counted(*args, **kwargs):
            if self.enabled:
                n = KERNELS_PER_CALL.get(name, 1)
                if name == "decode_attention" and kwargs.get("phase", 0) != 0:
                    n = 1  # one phase of a split launch: the attention splits or the merge
                self.launches += n
                self.calls[name] = self.calls.get(name, 0) + 1
            return fn(*args, **kwargs)

        return counted

    def reset(self) -> None:
        self.launches = 0
        self.calls = {}


_counter: LaunchCounter | None = None


def add_launches(name: str, count: int) -> None:
    """Record ``count`` kernel launches made inside one native call (e.g. the block-stack executor)."""
    if _counter is not None and _counter.enabled:
        _counter.launches += count
        _counter.calls[name] = _counter.calls.get(name, 0) + 1


def cutlass_include_dirs() -> list[str]:
    """CUTLASS/CuTe header trees shipped inside site-packages (used with -I only)."""
    site = Path(sysconfig.get_paths()["purelib"])
    for base in (site / "flashinfer" / "data" / "cutlass", site / "tilelang" / "3rdparty" / "cutlass"):
        if (base / "include" / "cutlass" / "cutlass.h").exists():
            return [str(base / "include"), str(base / "tools" / "util" / "include")]
    raise RuntimeError("CUTLASS headers not found (expected under flashinfer/data/cutlass)")


def _so_path() -> Path | None:
    suffix = importlib.machinery.EXTENSION_SUFFIXES
    for candidate in BUILD_DIR.glob(f"{NAME}*.so"):
        return candidate
    del suffix
    return None


def build(verbose: bool = False):
    """Compile (incrementally) and import the extension."""
    global _module
    from torch.utils import cpp_extension

    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    os.environ.setdefault("MAX_JOBS", str(max(os.cpu_count() or 4, 4)))
    cuda_flags = [*ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-DNDEBUG",
                  "-diag-suppress", "20012,177,550", "-DCUTLASS_ENABLE_DIRECT_CUDA_DRIVER_CALL=1", "-Xptxas", "-v" if verbose else "-O3"]
    _module = cpp_extension.load(
        name=NAME,
        sources=[str(CSRC / s) for s in _SOURCES],
        extra_include_paths=[str(CSRC), *cutlass_include_dirs()],
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=cuda_flags,
        build_directory=str(BUILD_DIR),
        verbose=verbose,
    )
    return _module


def load():
    """Import the built extension (no compilation); returns ``None`` when absent."""
    global _module
    if _module is not None:
        return _module
    if NAME in sys.modules:
        _module = sys.modules[NAME]
        return _module
    so = _so_path()
    if so is None:
        return None
    import torch  # noqa: F401  (the extension links against libtorch)

    spec = importlib.util.spec_from_file_location(NAME, str(so))
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    sys.modules[NAME] = module
    _module = module
    return module


def require():
    """The extension, or a clear error: CUDA tensors never take a silent fallback."""
    global _counter
    if _counter is not None:
        return _counter
    module = load()
    if module is None:
        raise RuntimeError(
            "The pra_ops CUDA extension is not built. Run `python -c 'import __graft_entry__ as g; g.build()'` "
            "(or pdattention_b200.ops._ext.build()) on a machine with nvcc before using CUDA tensors.")
    impl = os.environ.get("PRA_ATTENTION_IMPL")
    if impl:  # "tcgen05" (default) or "mma": which forward attention kernel runs
        module.set_attention_impl(impl)
    if os.environ.get("PRA_BOUNDS_CHECK", "0") == "1":  # bounds-checked gather / routing kernels
        module.set_bounds_check(True)
    if os.environ.get("PRA_DECODE_TMA", "1") == "0":  # the cp.async decode attention kernel
        module.decode_set_tma(False)
    if os.environ.get("PRA_PDL", "1") == "0":  # decode chain without programmatic dependent launch
        module.set_pdl(False)
    if os.environ.get("PRA_DG_CTAS") or os.environ.get("PRA_DG_MIN_KB") or os.environ.get("PRA_DG_MAX_SPLITS"):
        module.decode_gemm_configure(int(os.environ.get("PRA_DG_CTAS", 2)), int(os.environ.get("PRA_DG_MIN_KB", 8)),
                                     int(os.environ.get("PRA_DG_MAX_SPLITS", 0)))  # decode GEMM launch shape
    if os.environ.get("PRA_DECODE_STAGES"):  # pipeline depth of the TMA-fed decode kernel
        module.decode_set_stages(int(os.environ["PRA_DECODE_STAGES"]))
    _counter = LaunchCounter(module)
    return _counter


def launch_counter() -> LaunchCounter:
    return require()


def available() -> bool:
    return load() is not None
