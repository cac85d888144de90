"""Fixed-point rows on the GPU: the encoder's bytes bit-exact against the
oracle through the C ABI, and the decode layer on activations far outside
the fp16 range (bf16 holds them; the reference computes them in fp32)."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

DT = {torch.float32: 0, torch.bfloat16: 1}


def _encode_gpu(x: torch.Tensor, G: int):
    from phantom_moe import _lib
    lib = _lib.load()
    rows, K = x.shape
    nbytes = lib.phmoe_fx_rows_size(rows, K, G)
    out = torch.zeros(nbytes, dtype=torch.uint8, device=x.device)
    _lib.call("phmoe_fx_rows", x.data_ptr(), DT[x.dtype], rows, K, G, out.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    raw = out.cpu().numpy()
    cbytes = rows * (K // G) * 8
    q = raw[:rows * K * 2].reshape(rows, 2 * K)
    consts = raw[nbytes - cbytes:].view(np.int32).reshape(rows, K // G, 2)
    return q, consts


@pytest.mark.parametrize("G", [32, 64])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fx_rows_bitexact(cuda_device, G, dtype):
    import phantom_moe as pm
    rows, K = 24, 1024
    g = torch.Generator(device="cpu").manual_seed(7)
    scales = torch.tensor([1.0, 1e-3, 1e5, 1e6, 3e-20, 7e25, 0.0, 2.5] * 3)[:, None]
    x = torch.randn(rows, K, generator=g) * scales
    x[3, 17] = 4e9        # an outlier in one group of a row
    x[8, :] = 1e-40       # subnormal in fp32 (0 in bf16)
    x = x.to(dtype)
    q, consts = _encode_gpu(x.to(cuda_device), G)
    _, _, q_ref, c_ref, bad = O.fx_encode_rows(x.float().numpy(), G)
    assert not bad.any()
    assert np.array_equal(q, q_ref), np.argwhere(q != q_ref)[:5]
    assert np.array_equal(consts, c_ref), np.argwhere(consts != c_ref)[:5]
    assert pm.load_library().phmoe_device_error(1) == 0


def test_fx_rows_flags_values_it_cannot_hold(cuda_device):
    import phantom_moe as pm
    x = torch.ones(4, 256)
    x[0, 3] = float("inf")
    x[1, 7] = float("nan")
    x[2, 9] = 1e36
    q, consts = _encode_gpu(x.to(cuda_device), 64)
    _, _, q_ref, c_ref, bad = O.fx_encode_rows(x.numpy(), 64)
    assert np.array_equal(q, q_ref) and np.array_equal(consts, c_ref)
    with pytest.raises(pm.DeviceError) as ei:
        pm.check_device_errors()
    assert ei.value.bits & 2
    pm.check_device_errors()  # cleared by the first read


@pytest.mark.parametrize("scale", [1e5, 1e6, 3e-6])
@pytest.mark.parametrize("T", [5, 64])
def test_decode_layer_activations_beyond_fp16(cuda_device, scale, T):
    """bf16 activations of magnitude 1e5-1e6 (and tiny ones): the SwiGLU
    output reaches ~1e12, far beyond fp16; the fixed-point rows give every
    group its own exponent, so the layer matches the fp32 oracle with the
    contract tolerance taken relative to the output's scale, and no error
    bit is raised."""
    import phantom_moe as pm
    dev = cuda_device
    E, H, k, I, G = 32, 1024, 4, 512, 64
    gen = torch.Generator(device=dev).manual_seed(11)
    wr = (torch.randn(E, H, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
    pk = pm.pack_experts(torch.randn(E, 2 * I, H, device=dev, generator=gen) * 0.02,
                         torch.randn(E, H, I, device=dev, generator=gen) * 0.02, G)
    x = (torch.randn(T, H, device=dev, generator=gen) * scale).to(torch.bfloat16)
    out, idx, w = pm.moe_layer(x, wr, pk.w13_q, pk.w13_scales, pk.w2_q, pk.w2_scales, k, group_size=G,
                               path="decode", return_routing=True, check_errors=True)
    host = [t.cpu().numpy() for t in (pk.w13_q, pk.w13_scales, pk.w2_q, pk.w2_scales)]
    ref, i_ref, _ = O.moe_layer_reference_packed(x.float().cpu().numpy(), wr.float().cpu().numpy(), *host, k, G)
    assert np.array_equal(idx.cpu().numpy(), i_ref)
    got = out.float().cpu().numpy()
    assert np.all(np.isfinite(got))
    ref_scale = float(np.abs(ref).max())
    mx, mr = O.parity_stats(got / ref_scale, ref / ref_scale)
    assert mx <= O.MAX_ABS_TOL and mr <= O.MEAN_REL_TOL, (mx, mr)
