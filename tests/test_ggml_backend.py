"""The ggml backend library (questwend_b200/libggml-qwb.so) on a host without a B200: it
loads against the reference's own ggml, exports ggml's dynamic-loader entry points,
registers an interface-version-3 registry named QWB, and reports score 0 and no devices,
so ggml_backend_load_all() on such a host skips it.  No GPU is used."""
import ctypes as C
import os

import numpy as np
import pytest

import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHIM = os.path.join(ROOT, "questwend_b200", "libggml-qwb.so")
HEADER = os.path.join(ROOT, "include", "qwb_ggml_backend.h")


@pytest.fixture(scope="module")
def shim():
    if not os.path.exists(SHIM):
        pytest.skip("libggml-qwb.so not built (needs the reference ggml headers)")
    if not O.ref_available():
        pytest.skip("the reference ggml (oracle/_ref) is not built")
    O.ref()  # ggml symbols the shim resolves at load time
    return C.CDLL(SHIM)


def test_exports_every_declared_entry_point(shim):
    text = open(HEADER).read()
    for name in ("ggml_backend_qwb_reg", "ggml_backend_init", "ggml_backend_score"):
        assert f"{name}(void)" in text
        assert hasattr(shim, name)


def test_registry_is_interface_version_3_named_QWB(shim):
    shim.ggml_backend_init.restype = C.c_void_p
    reg = shim.ggml_backend_init()
    assert reg
    assert C.c_int.from_address(reg).value == 3  # struct ggml_backend_reg.api_version
    ref = O.ref()
    ref.ggml_backend_reg_name.restype = C.c_char_p
    ref.ggml_backend_reg_name.argtypes = [C.c_void_p]
    assert ref.ggml_backend_reg_name(reg) == b"QWB"
    ref.ggml_backend_reg_dev_count.restype = C.c_size_t
    ref.ggml_backend_reg_dev_count.argtypes = [C.c_void_p]
    shim.ggml_backend_qwb_reg.restype = C.c_void_p
    assert shim.ggml_backend_qwb_reg() == reg


def test_no_b200_means_score_0_and_no_device(shim):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    assert shim.ggml_backend_score() == 0
    # ggml's own loader (ggml_backend_load) checks the score and declines the library
    w = np.zeros(O.row_size(O.Q8_0, 64) * 4, dtype=np.uint8)
    _, rc = O.backend_mul_mat_id(SHIM, O.Q8_0, w, 64, 2, 2, np.zeros((1, 1, 64), np.float32),
                                 np.zeros((1, 2), np.int32))
    assert rc == -1


def test_mul_mat_reference_driver_matches_restatement():
    # the reference's own ggml_mul_mat (CPU backend) and the restatement agree; the GPU
    # tests hold qwb_mul_mat to the former
    if not O.ref_available():
        pytest.skip("the reference ggml (oracle/_ref) is not built")
    import _data as D
    for t, K, M, T in ((O.Q4_K, 512, 96, 5), (O.Q6_K, 768, 64, 9), (O.Q8_0, 256, 40, 3)):
        w = D.weights(t, 1, M, K, seed=K)
        b = D.acts((T, K), seed=T)
        r, _ = O.mul_mat(t, w, K, M, b, impl="ref")
        p, rc = O.mul_mat(t, w, K, M, b)
        assert rc == 0 and O.nrmse(p, r) <= 1e-6
