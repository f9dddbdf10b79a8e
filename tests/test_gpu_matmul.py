"""Op sweep of the ternary matmul: the 2B layer shapes at M from 1 to 4096
(every C2 cell: M in {1, 8, 64, 512, 4096}) plus edge sizes, through the
device-resident C-ABI entry points.  Int8 activations and int32
accumulators must be bit-exact; f32 outputs bit-exact against the oracle's
ternary_gemv_quantised applied per row."""
import ctypes as C

import numpy as np
import pytest

import oracle_lib as O
from bitnetrs_b200 import _native as N
from bitnetrs_b200 import synth

pytestmark = pytest.mark.gpu
L = O.lib()


def unpack_codes(packed, rows, cols):
    pc = (cols + 3) // 4
    b = packed.reshape(rows, pc)
    codes = np.stack([(b >> (2 * j)) & 3 for j in range(4)], axis=-1).reshape(rows, pc * 4)[:, :cols]
    return np.where(codes == 0, 1.0, np.where(codes == 2, -1.0, 0.0))


@pytest.mark.parametrize("M", [1, 2, 8, 16, 17, 64, 65, 128, 200, 256, 512, 1000, 4096])
@pytest.mark.parametrize("N_,K", [(2560, 2560), (640, 2560), (2560, 6912), (6912, 2560), (100, 200)])
def test_device_matmul_bit_exact(cuda_backend, M, N_, K):
    import torch

    lib = N.cuda_lib()
    dev = torch.device("cuda", cuda_backend.device_id)
    packed = synth.ternary_codes(M + N_, 3, N_, K)
    scale = 0.0161
    wh = C.c_void_p()
    N.check(lib.bitnet_cuda_weight_upload(cuda_backend.handle, packed.ctypes.data, packed.size, N_, K, scale,
                                          C.byref(wh)))
    x_bf16 = synth.bf16_normal(M, 7, M * K, 1.0)
    ldq = (K + 63) // 64 * 64
    d_x = torch.from_numpy(x_bf16.view(np.int16).copy()).to(dev)
    d_xq = torch.zeros((M, ldq), dtype=torch.int8, device=dev)
    d_amax = torch.zeros(M, dtype=torch.float32, device=dev)
    d_rs = torch.zeros(M, dtype=torch.int32, device=dev)
    d_st = torch.zeros(1, dtype=torch.int32, device=dev)
    d_out = torch.zeros((M, N_), dtype=torch.float32, device=dev)
    d_acc = torch.zeros((M, N_), dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    N.check(lib.bitnet_cuda_quantize_rows_device(cuda_backend.handle, d_x.data_ptr(), 1, M, K, d_xq.data_ptr(), ldq,
                                                 d_amax.data_ptr(), d_rs.data_ptr(), d_st.data_ptr(), None))
    N.check(lib.bitnet_cuda_ternary_matmul_device(cuda_backend.handle, wh, d_xq.data_ptr(), ldq, d_amax.data_ptr(),
                                                  d_rs.data_ptr(), M, d_out.data_ptr(), d_acc.data_ptr(), None))
    torch.cuda.synchronize()
    lib.bitnet_cuda_weight_destroy(wh)
    xq = d_xq.cpu().numpy()[:, :K]
    amax = d_amax.cpu().numpy()
    assert d_st.item() == 0
    # int8 activations: the reference quantiser on the same rows
    xf = synth.bf16_bits_to_f32(x_bf16).reshape(M, K)
    for m in range(0, M, max(1, M // 8)):
        q = np.zeros(K, dtype=np.int8)
        s = C.c_float()
        assert L.orc_absmax_quantize_row_into(O.p(xf[m].copy()), K, O.p(q), K, C.byref(s)) == 0
        np.testing.assert_array_equal(xq[m], q)
        assert amax[m] == np.float32(s.value) * np.float32(127.0)
    # int32 accumulators: exact integer product (float64 is exact at these magnitudes)
    W = unpack_codes(packed, N_, K)
    ref_acc = (xq.astype(np.float64) @ W.T).astype(np.int64)
    np.testing.assert_array_equal(d_acc.cpu().numpy(), ref_acc)
    # f32 outputs: the reference epilogue per row
    out = d_out.cpu().numpy()
    for m in range(0, M, max(1, M // 4)):
        ro = np.zeros(N_, dtype=np.float32)
        assert L.orc_ternary_gemv_preq(O.p(packed), packed.size, scale, O.p(np.ascontiguousarray(xq[m])), K,
                                       float(amax[m]), O.p(ro), N_, N_, K, None) == 0
        np.testing.assert_array_equal(out[m], ro)


@pytest.mark.parametrize("N_,K", [(3840, 2560), (13824, 2560), (2560, 6912), (4096, 14336), (96, 20480), (33, 64)])
def test_decode_gemv_bit_exact(cuda_backend, N_, K):
    """M = 1 (decode) at the fused 2B shapes (qkv, gate|up), the 2B and
    scaled-model down projections and rows past the shared-memory x stage."""
    import torch

    lib = N.cuda_lib()
    dev = torch.device("cuda", cuda_backend.device_id)
    packed = synth.ternary_codes(N_ + K, 5, N_, K)
    scale = 0.0123
    wh = C.c_void_p()
    N.check(lib.bitnet_cuda_weight_upload(cuda_backend.handle, packed.ctypes.data, packed.size, N_, K, scale,
                                          C.byref(wh)))
    ldq = (K + 63) // 64 * 64
    x_bf16 = synth.bf16_normal(K, 9, K, 1.0)
    d_x = torch.from_numpy(x_bf16.view(np.int16).copy()).to(dev)
    d_xq = torch.zeros((1, ldq), dtype=torch.int8, device=dev)
    d_amax = torch.zeros(1, dtype=torch.float32, device=dev)
    d_rs = torch.zeros(1, dtype=torch.int32, device=dev)
    d_st = torch.zeros(1, dtype=torch.int32, device=dev)
    d_out = torch.zeros((1, N_), dtype=torch.float32, device=dev)
    d_acc = torch.zeros((1, N_), dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    N.check(lib.bitnet_cuda_quantize_rows_device(cuda_backend.handle, d_x.data_ptr(), 1, 1, K, d_xq.data_ptr(), ldq,
                                                 d_amax.data_ptr(), d_rs.data_ptr(), d_st.data_ptr(), None))
    N.check(lib.bitnet_cuda_ternary_matmul_device(cuda_backend.handle, wh, d_xq.data_ptr(), ldq, d_amax.data_ptr(),
                                                  d_rs.data_ptr(), 1, d_out.data_ptr(), d_acc.data_ptr(), None))
    torch.cuda.synchronize()
    lib.bitnet_cuda_weight_destroy(wh)
    xq = d_xq.cpu().numpy()[:, :K]
    W = unpack_codes(packed, N_, K)
    np.testing.assert_array_equal(d_acc.cpu().numpy(), (xq.astype(np.float64) @ W.T).astype(np.int64))
    ro = np.zeros(N_, dtype=np.float32)
    assert L.orc_ternary_gemv_preq(O.p(packed), packed.size, scale, O.p(np.ascontiguousarray(xq[0])), K,
                                   float(d_amax.item()), O.p(ro), N_, N_, K, None) == 0
    np.testing.assert_array_equal(d_out.cpu().numpy()[0], ro)


@pytest.mark.parametrize("N_,K", [(40000, 2560), (38000, 6912), (40001, 2048)])
def test_decode_gemv_many_rows_bit_exact(cuda_backend, N_, K):
    """M = 1 over tens of thousands of rows (the shape of the bench's
    gemv_stream, every layer's weights of one input width in one launch):
    int32 accumulators and f32 outputs equal to the oracle's
    ternary_gemv_quantised."""
    import torch

    lib = N.cuda_lib()
    dev = torch.device("cuda", cuda_backend.device_id)
    packed = synth.ternary_codes(N_ + K, 6, N_, K)
    scale = 0.0117
    wh = C.c_void_p()
    N.check(lib.bitnet_cuda_weight_upload(cuda_backend.handle, packed.ctypes.data, packed.size, N_, K, scale,
                                          C.byref(wh)))
    ldq = (K + 63) // 64 * 64
    x_bf16 = synth.bf16_normal(K, 10, K, 1.0)
    d_x = torch.from_numpy(x_bf16.view(np.int16).copy()).to(dev)
    d_xq = torch.zeros((1, ldq), dtype=torch.int8, device=dev)
    d_amax = torch.zeros(1, dtype=torch.float32, device=dev)
    d_rs = torch.zeros(1, dtype=torch.int32, device=dev)
    d_st = torch.zeros(1, dtype=torch.int32, device=dev)
    d_out = torch.zeros((1, N_), dtype=torch.float32, device=dev)
    d_acc = torch.zeros((1, N_), dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    N.check(lib.bitnet_cuda_quantize_rows_device(cuda_backend.handle, d_x.data_ptr(), 1, 1, K, d_xq.data_ptr(), ldq,
                                                 d_amax.data_ptr(), d_rs.data_ptr(), d_st.data_ptr(), None))
    N.check(lib.bitnet_cuda_ternary_matmul_device(cuda_backend.handle, wh, d_xq.data_ptr(), ldq, d_amax.data_ptr(),
                                                  d_rs.data_ptr(), 1, d_out.data_ptr(), d_acc.data_ptr(), None))
    torch.cuda.synchronize()
    lib.bitnet_cuda_weight_destroy(wh)
    xq = np.ascontiguousarray(d_xq.cpu().numpy()[0, :K])
    ro = np.zeros(N_, dtype=np.float32)
    racc = np.zeros(N_, dtype=np.int32)
    assert L.orc_ternary_gemv_preq(O.p(packed), packed.size, scale, O.p(xq), K, float(d_amax.item()), O.p(ro), N_,
                                   N_, K, O.p(racc)) == 0
    np.testing.assert_array_equal(d_acc.cpu().numpy()[0], racc)
    np.testing.assert_array_equal(d_out.cpu().numpy()[0], ro)


# The per-rank projection shapes of the scaled model split over 2, 4 and 8
# tensor-parallel ranks (q/k/v and gate/up by rows, o and down by columns),
# at the decode batch of C5 and at one row.
TP_SHAPES = sorted({(N_, K) for w in (2, 4, 8) for N_, K in (
    ((32 // w + 2 * (8 // w)) * 128, 4096), (4096, 32 // w * 128), (2 * 14336 // w, 4096), (4096, 14336 // w))})


@pytest.mark.parametrize("M", [1, 64])
@pytest.mark.parametrize("N_,K", TP_SHAPES)
def test_device_matmul_tp_rank_shapes(cuda_backend, M, N_, K):
    test_device_matmul_bit_exact(cuda_backend, M, N_, K)
