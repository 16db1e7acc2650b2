"""A failed argument check inside the compiled extension raises a Python error.

The extension links the shared libstdc++ that libtorch uses; a private static
copy left its stream state unset, so formatting an error message, on the
autograd engine's worker threads as on any other, crashed the process instead of
raising.
"""
import threading

import pytest
import torch


def _ext():
    from complexity_framework_b200.ops import load

    C = load()
    if C is None:
        pytest.skip("extension not built")
    return C


def _bad_call(C):
    z = torch.zeros(1, 1, 8, 64)
    C.flash_attn_fwd(z.bfloat16(), z, z, torch.zeros(1), torch.zeros(1), 1.0, True)


def test_argument_check_raises_on_main_thread():
    C = _ext()
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        _bad_call(C)


def test_argument_check_raises_on_worker_thread():
    C = _ext()
    seen = []

    def run():
        try:
            _bad_call(C)
        except RuntimeError as exc:
            seen.append(str(exc))

    t = threading.Thread(target=run)
    t.start()
    t.join()
    assert seen and "must be a CUDA tensor" in seen[0]
