"""Host behaviour of the reference-mirroring API: validation messages follow
the reference binding, and without a GPU the compute calls raise (there is
no CPU fallback)."""
import numpy as np
import pytest
import torch

from siliconfer_b200.kernels import cuda as K


def test_api_names_mirror_reference():
    for name in ("pack_weights_sym", "pack_weights_asym", "gemv_sym", "gemv_scalar",
                 "gemv_asym", "gemm_sym", "gemm_asym"):
        assert callable(getattr(K, name))


@pytest.mark.parametrize("call,msg", [
    (lambda: K.gemv_sym(np.zeros((4,), np.uint8), np.zeros((4, 1), np.float32),
                        np.zeros(8, np.float32), 8), "W must be 2-D"),
    (lambda: K.gemv_sym(np.zeros((4, 4), np.uint8), np.zeros((4,), np.float32),
                        np.zeros(8, np.float32), 8), "scales must be 2-D"),
    (lambda: K.gemv_sym(np.zeros((4, 4), np.uint8), np.zeros((4, 2), np.float32),
                        np.zeros(8, np.float32), 8), "scales shape mismatch"),
    (lambda: K.gemv_sym(np.zeros((4, 4), np.uint8), np.zeros((4, 1), np.float32),
                        np.zeros(7, np.float32), 8), "x length mismatch"),
    (lambda: K.gemv_sym(np.zeros((4, 4), np.uint8), np.zeros((4, 1), np.float32),
                        np.zeros((1, 8), np.float32), 8), "x must be 1-D"),
    (lambda: K.gemm_sym(np.zeros((4, 4), np.uint8), np.zeros((4, 1), np.float32),
                        np.zeros((2, 7), np.float32), 8), "X/W in_features mismatch"),
    (lambda: K.gemm_asym(np.zeros((4, 4), np.uint8), np.zeros((4, 1), np.float32),
                         np.zeros((4, 2), np.float32), np.zeros((2, 8), np.float32), 8),
     "zeros shape mismatch"),
])
def test_validation_messages(call, msg):
    with pytest.raises(RuntimeError, match=msg):
        call()


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
def test_no_cpu_fallback():
    assert not K.CUDA_AVAILABLE
    p, s = K.pack_weights_sym(np.ones((4, 64), np.float32), 64)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        K.gemv_sym(p, s, np.ones(64, np.float32), 64)
