"""The op-level drop-in: the reference's own model loop over this library's
CUDA backend for its op API.

oracle/_ref/libtorchless_ref_cuda.so is the reference's src/common/tensor.cpp,
src/loader/parameters.cpp, src/model/mistral/modules.cpp and main.cpp,
compiled unchanged together with torchless_b200/backend_cuda/kernels.cpp in
place of src/backend/cpu/kernels.cpp (oracle/Makefile, target ref-cuda).  Every
kernels.h op of Model<int8_t>::forward (modules.cpp:154-171) then runs on the
GPU through the C ABI.  The TINY golden model, loaded from a file through the
reference's own loader, must reproduce the reference's greedy fixture
(tests/golden/ref_greedy_tiny.npz): logits within the op tolerance, ids
identical (near-tie rule of the model tests).
"""
import os

import numpy as np
import pytest

from conftest import golden_greedy, rel_err

import oracle

SYMBOLS = ["ref_load_file", "ref_load_buffer", "ref_forward", "ref_logits", "ref_sample_max", "ref_free"]


def test_dropin_library_links_the_cuda_backend():
    """Built (where the reference tree was present) and resolvable without a GPU."""
    if not oracle.ref_cuda_available():
        pytest.skip("oracle/_ref/libtorchless_ref_cuda.so not built here")
    L = oracle.ref_cuda_lib()
    for name in SYMBOLS:
        assert getattr(L, name) is not None


@pytest.mark.gpu
def test_reference_model_loop_over_cuda_ops(tiny_bin, tmp_path):
    torch = pytest.importorskip("torch")
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    assert oracle.ref_cuda_available(), "oracle/_ref/libtorchless_ref_cuda.so is missing"
    path = os.path.join(tmp_path, "tiny.bin")
    np.asarray(tiny_bin).tofile(path)
    prompt, ids, logits = golden_greedy("tiny")
    rm = oracle.RefModel(path=path, max_seq=64, lib=oracle.ref_cuda_lib())
    for t in prompt[:-1]:
        rm.forward(int(t))
    feed = [prompt[-1]] + list(ids[:-1])
    worst, ties = 0.0, []
    for step, tok in enumerate(feed):
        lg = rm.forward(int(tok))
        e = rel_err(lg, logits[step])
        worst = max(worst, e)
        assert e <= 1e-4, f"step {step}: logits rel err {e}"
        got = rm.sample_max()
        if got != ids[step]:
            top = np.sort(logits[step])[-2:]
            assert (top[1] - top[0]) < 1e-3 * np.max(np.abs(logits[step])), f"step {step}: {got} != {ids[step]}"
            ties.append(step)
    rm.close()
    print(f"reference loop over CUDA ops: {len(feed)} steps, worst rel err {worst:.2e}, near-ties {ties}")
