"""Device policy: which device runs, whether the native sm_100a kernels run,
and small helpers around them.

Counterpart of complexity/utils/device.py:30-330.  The reference chooses among
CUDA, ROCm, MPS and CPU and gates its Triton kernels per backend; this
framework is written for one GPU target, so the backends are NVIDIA CUDA
(the native kernels of ``complexity_framework_b200._C`` run when the GPU is
sm_100 and the extension is built) and CPU (PyTorch reference paths).  The
ROCm and MPS queries exist for callers that ask; they report unavailable.
"""
from __future__ import annotations

import logging
import os
import random
from contextlib import contextmanager, nullcontext
from dataclasses import asdict, dataclass
from typing import Literal, Optional, Union

import torch

logger = logging.getLogger(__name__)

BackendName = Literal["cuda", "cpu"]
KernelPolicy = Union[Literal["auto"], bool]


@dataclass(frozen=True)
class BackendInfo:
    name: str
    device: torch.device
    device_name: str
    compute_capability: Optional[str] = None
    custom_kernels: bool = False
    sdpa: bool = False
    matmul: str = "cpu"
    distributed: str = "gloo"


def is_nvidia_cuda_available() -> bool:
    return torch.cuda.is_available() and torch.version.hip is None


def is_mps_available() -> bool:
    return False  # not a target of this framework


def is_rocm_available() -> bool:
    return False  # not a target of this framework


def is_rocm_runtime_present() -> bool:
    return False


def rocm_unavailable_message() -> str:
    return ("this framework targets NVIDIA B200 (sm_100a) GPUs; ROCm devices are not supported. "
            "Run on CUDA or on the CPU reference paths.")


def get_backend(preferred: str = "auto") -> str:
    p = (preferred or "auto").lower()
    if p in ("rocm", "hip", "mps"):
        raise RuntimeError(rocm_unavailable_message() if p != "mps" else
                           "Apple MPS is not a target of this framework; use cuda or cpu")
    if p == "cuda":
        if not is_nvidia_cuda_available():
            raise RuntimeError("CUDA was requested but no NVIDIA GPU is visible")
        return "cuda"
    if p == "cpu":
        return "cpu"
    if p != "auto":
        raise ValueError(f"unknown backend {preferred!r}")
    return "cuda" if is_nvidia_cuda_available() else "cpu"


def select_device(preferred: str = "auto") -> torch.device:
    b = get_backend(preferred)
    return torch.device("cuda", torch.cuda.current_device()) if b == "cuda" else torch.device("cpu")


def _capability(device: torch.device) -> Optional[str]:
    if device.type != "cuda":
        return None
    major, minor = torch.cuda.get_device_capability(device)
    return f"{major}.{minor}"


def custom_kernels_enabled(policy: KernelPolicy = "auto") -> bool:
    """Whether the native kernels run: policy ``False`` (or the environment
    variable ``COMPLEXITY_USE_CUSTOM_KERNELS=0``) turns them off; ``True``
    demands them (an error when they cannot run); ``auto`` uses them on an
    sm_100 GPU with the extension built."""
    env = os.environ.get("COMPLEXITY_USE_CUSTOM_KERNELS")
    if env is not None and policy == "auto":
        policy = env.strip().lower() not in ("0", "false", "no", "off")
    if policy is False:
        return False
    ok = False
    if is_nvidia_cuda_available():
        from ..ops import available

        ok = available() and torch.cuda.get_device_capability()[0] == 10
    if policy is True and not ok:
        raise RuntimeError("custom kernels were requested but need an sm_100 GPU and the built "
                           "extension (python __graft_entry__.py build, or setup.py build_ext)")
    return ok


def supports_custom_triton(policy: KernelPolicy = "auto") -> bool:
    """The reference's Triton gate; the hot ops here are CUDA C++, so this is
    the same question as ``custom_kernels_enabled``."""
    return custom_kernels_enabled(policy)


def get_backend_info(preferred: str = "auto", kernel_policy: KernelPolicy = "auto") -> BackendInfo:
    dev = select_device(preferred)
    if dev.type == "cuda":
        return BackendInfo(name="cuda", device=dev, device_name=torch.cuda.get_device_name(dev),
                           compute_capability=_capability(dev),
                           custom_kernels=custom_kernels_enabled(kernel_policy), sdpa=True,
                           matmul="tcgen05" if custom_kernels_enabled(kernel_policy) else "cublas",
                           distributed="nccl")
    return BackendInfo(name="cpu", device=dev, device_name="cpu", sdpa=True)


def log_backend(preferred: str = "auto", kernel_policy: KernelPolicy = "auto") -> BackendInfo:
    info = get_backend_info(preferred, kernel_policy)
    logger.info("backend=%s device=%s (%s) cc=%s custom_kernels=%s distributed=%s", info.name,
                info.device, info.device_name, info.compute_capability, info.custom_kernels,
                info.distributed)
    return info


def backend_metadata(preferred: str = "auto", kernel_policy: KernelPolicy = "auto") -> dict:
    d = asdict(get_backend_info(preferred, kernel_policy))
    d["device"] = str(d["device"])
    d["torch"] = torch.__version__
    d["cuda"] = torch.version.cuda
    return d


def configure_torch_acceleration(kernel_policy: KernelPolicy = "auto",
                                 log: bool = True) -> BackendInfo:
    """TF32 for fp32 matmuls / convolutions and cuDNN autotuning on CUDA."""
    if is_nvidia_cuda_available():
        torch.backends.cuda.matmul.allow_tf32 = True
        torch.backends.cudnn.allow_tf32 = True
        torch.backends.cudnn.benchmark = True
    return log_backend("auto", kernel_policy) if log else get_backend_info("auto", kernel_policy)


_SDPA = {"flash": "FLASH_ATTENTION", "efficient": "EFFICIENT_ATTENTION", "math": "MATH",
         "cudnn": "CUDNN_ATTENTION"}


def sdpa_kernel_backends():
    """SDPA backends from ``COMPLEXITY_SDPA_BACKENDS`` (comma list of flash,
    efficient, math, cudnn) for the module paths that still call SDPA; None =
    PyTorch's choice."""
    names = os.environ.get("COMPLEXITY_SDPA_BACKENDS")
    if not names:
        return None
    from torch.nn.attention import SDPBackend

    out = []
    for n in names.split(","):
        n = n.strip().lower()
        if n not in _SDPA:
            raise ValueError(f"unknown SDPA backend {n!r}; choose from {sorted(_SDPA)}")
        out.append(getattr(SDPBackend, _SDPA[n]))
    return out


def sdpa_kernel_context():
    b = sdpa_kernel_backends()
    if b is None:
        return nullcontext()
    from torch.nn.attention import sdpa_kernel

    return sdpa_kernel(b)


def empty_cache(device: torch.device) -> None:
    if torch.device(device).type == "cuda":
        torch.cuda.empty_cache()


def synchronize(device: torch.device) -> None:
    if torch.device(device).type == "cuda":
        torch.cuda.synchronize(device)


def seed_all(seed: int) -> None:
    random.seed(seed)
    try:
        import numpy as np

        np.random.seed(seed % (2 ** 32))
    except ImportError:  # pragma: no cover
        pass
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)


def autocast_dtype(device: torch.device, prefer_bf16: bool = True) -> Optional[torch.dtype]:
    """bf16 on CUDA (fp16 when bf16 is not preferred); no autocast on CPU."""
    if torch.device(device).type != "cuda":
        return None
    return torch.bfloat16 if prefer_bf16 else torch.float16


@contextmanager
def autocast(device: torch.device, dtype: Optional[torch.dtype] = None, enabled: bool = True):
    dev = torch.device(device)
    dt = dtype or autocast_dtype(dev)
    if not enabled or dt is None:
        yield
        return
    with torch.autocast(dev.type, dtype=dt):
        yield
