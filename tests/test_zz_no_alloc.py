"""bitnet_cuda_ternary_gemv_quant_noalloc against the allocating device path.

The no-alloc entry point keeps its activation scratch in a fixed device array
of the library; it must give the same outputs as quantize_rows_device +
ternary_matmul_device (bit-exact, so the tolerance is 0) on two calls in a
row, reject rows longer than its scratch and report non-finite input.  This
file is collected last so it also runs after every other GPU test."""
import ctypes as C

import numpy as np
import pytest

from bitnetrs_b200 import _native as N
from bitnetrs_b200 import synth
from bitnetrs_b200.errors import InvalidShape, QuantizationError

pytestmark = pytest.mark.gpu


def _upload(be, n, k, seed):
    packed = synth.ternary_codes(seed, 4, n, k)
    wh = C.c_void_p()
    N.check(N.cuda_lib().bitnet_cuda_weight_upload(be.handle, packed.ctypes.data, packed.size, n, k, 0.0173,
                                                    C.byref(wh)))
    return wh


def _reference(be, wh, d_x, n, k, dev):
    import torch

    lib = N.cuda_lib()
    ldq = (k + 63) // 64 * 64
    d_xq = torch.zeros(ldq, dtype=torch.int8, device=dev)
    d_amax = torch.zeros(1, dtype=torch.float32, device=dev)
    d_rs = torch.zeros(1, dtype=torch.int32, device=dev)
    d_st = torch.zeros(1, dtype=torch.int32, device=dev)
    d_out = torch.zeros(n, dtype=torch.float32, device=dev)
    N.check(lib.bitnet_cuda_quantize_rows_device(be.handle, d_x.data_ptr(), 0, 1, k, d_xq.data_ptr(), ldq,
                                                 d_amax.data_ptr(), d_rs.data_ptr(), d_st.data_ptr(), None))
    N.check(lib.bitnet_cuda_ternary_matmul_device(be.handle, wh, d_xq.data_ptr(), ldq, d_amax.data_ptr(),
                                                  d_rs.data_ptr(), 1, d_out.data_ptr(), None, None))
    torch.cuda.synchronize()
    assert d_st.item() == 0
    return d_out.cpu().numpy()


@pytest.mark.parametrize("n,k", [(2560, 2560), (3840, 2560), (2560, 6912), (100, 200), (64, 32768)])
def test_noalloc_matches_device_path_twice(cuda_backend, n, k):
    import torch

    lib = N.cuda_lib()
    dev = torch.device("cuda", cuda_backend.device_id)
    wh = _upload(cuda_backend, n, k, n + k)
    x = synth.bf16_bits_to_f32(synth.bf16_normal(k, 3, k, 1.0)).astype(np.float32)
    d_x = torch.from_numpy(x).to(dev)
    ref = _reference(cuda_backend, wh, d_x, n, k, dev)
    for _ in range(2):
        d_out = torch.full((n,), float("nan"), dtype=torch.float32, device=dev)
        torch.cuda.synchronize()
        N.check(lib.bitnet_cuda_ternary_gemv_quant_noalloc(cuda_backend.handle, wh, d_x.data_ptr(), k,
                                                           d_out.data_ptr(), n, None))
        np.testing.assert_allclose(d_out.cpu().numpy(), ref, rtol=0, atol=0)
    lib.bitnet_cuda_weight_destroy(wh)


def test_noalloc_rejects_long_rows_and_non_finite(cuda_backend):
    import torch

    lib = N.cuda_lib()
    dev = torch.device("cuda", cuda_backend.device_id)
    k_long = 32768 + 64
    wh = _upload(cuda_backend, 8, k_long, 1)
    d_x = torch.zeros(k_long, dtype=torch.float32, device=dev)
    d_out = torch.zeros(8, dtype=torch.float32, device=dev)
    with pytest.raises(InvalidShape):
        N.check(lib.bitnet_cuda_ternary_gemv_quant_noalloc(cuda_backend.handle, wh, d_x.data_ptr(), k_long,
                                                           d_out.data_ptr(), 8, None))
    lib.bitnet_cuda_weight_destroy(wh)
    wh = _upload(cuda_backend, 8, 256, 2)
    x = np.ones(256, dtype=np.float32)
    x[17] = np.inf
    d_x = torch.from_numpy(x).to(dev)
    with pytest.raises(QuantizationError):
        N.check(lib.bitnet_cuda_ternary_gemv_quant_noalloc(cuda_backend.handle, wh, d_x.data_ptr(), 256,
                                                           d_out.data_ptr(), 8, None))
    # the flag does not stick: a finite row after the failure succeeds
    d_x = torch.ones(256, dtype=torch.float32, device=dev)
    N.check(lib.bitnet_cuda_ternary_gemv_quant_noalloc(cuda_backend.handle, wh, d_x.data_ptr(), 256,
                                                       d_out.data_ptr(), 8, None))
    lib.bitnet_cuda_weight_destroy(wh)
