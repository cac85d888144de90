"""HostPipeline: pinned host batches through MoE layers with the copies on
their own streams give the bits of the synchronous per-step calls."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _layers(dev, n, E=32, H=1024, I=256, k=4, G=64):
    import phantom_moe as pm
    out = []
    for l in range(n):
        gen = torch.Generator(device=dev).manual_seed(70 + l)
        pk = pm.pack_experts(torch.randn(E, 2 * I, H, device=dev, generator=gen) * 0.02,
                             torch.randn(E, H, I, device=dev, generator=gen) * 0.02, G)
        wr = (torch.randn(E, H, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
        out.append(pm.MoeLayer(wr, pk.w13_q, pk.w13_scales, pk.w2_q, pk.w2_scales, k, group_size=G))
    return out


@pytest.mark.parametrize("depth", [1, 2, 3])
def test_pipeline_matches_synchronous_calls(cuda_device, depth):
    import phantom_moe as pm
    dev, T, H = cuda_device, 40, 1024
    layers = _layers(dev, 3)
    pipe = pm.HostPipeline(layers, T, H, device=dev, depth=depth)
    steps = 7
    g = torch.Generator().manual_seed(5)
    xh = [torch.randn(T, H, generator=g).to(torch.bfloat16).pin_memory() for _ in range(steps)]
    oh = [torch.empty(T, H, dtype=torch.bfloat16).pin_memory() for _ in range(steps)]
    for i in range(steps):
        pipe.submit(xh[i], oh[i])
    pipe.synchronize()
    for i in range(steps):
        ref = layers[i % 3](xh[i].to(dev)).cpu()
        assert torch.equal(oh[i], ref), i


def test_pipeline_reused_host_buffers_and_eager_callables(cuda_device):
    """Host buffers reused once their step's event completes; a plain
    callable runs eagerly on the compute stream."""
    import phantom_moe as pm
    dev, T, H = cuda_device, 24, 1024
    layer = _layers(dev, 1)[0]
    pipe = pm.HostPipeline([lambda x, out: layer(x, out=out)], T, H, device=dev)
    g = torch.Generator().manual_seed(9)
    xs = [torch.randn(T, H, generator=g).to(torch.bfloat16) for _ in range(5)]
    xh = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()
    oh = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()
    for x in xs:
        xh.copy_(x)
        pipe.submit(xh, oh).synchronize()
        assert torch.equal(oh, layer(x.to(dev)).cpu())


def test_pipeline_step_events_stay_valid(cuda_device):
    """The event submit() returns belongs to its step: waiting on it after
    later steps have reused the same device slot still means that step's
    result is on the host."""
    import phantom_moe as pm
    dev, T, H, depth = cuda_device, 16, 1024, 2
    layers = _layers(dev, 1)
    pipe = pm.HostPipeline(layers, T, H, device=dev, depth=depth)
    g = torch.Generator().manual_seed(13)
    steps = 2 * depth + 1
    xh = [torch.randn(T, H, generator=g).to(torch.bfloat16).pin_memory() for _ in range(steps)]
    oh = [torch.empty(T, H, dtype=torch.bfloat16).pin_memory() for _ in range(steps)]
    evs = [pipe.submit(xh[i], oh[i]) for i in range(steps)]
    assert len({id(e) for e in evs}) == steps
    evs[0].synchronize()
    assert torch.equal(oh[0], layers[0](xh[0].to(dev)).cpu())
    pipe.synchronize()
    assert all(e.query() for e in evs)


def test_pipeline_rejects_bad_buffers(cuda_device):
    import phantom_moe as pm
    dev = cuda_device
    pipe = pm.HostPipeline(_layers(dev, 1), 8, 1024, device=dev)
    ok = torch.empty(8, 1024, dtype=torch.bfloat16).pin_memory()
    with pytest.raises(ValueError):
        pipe.submit(torch.empty(8, 1024, dtype=torch.bfloat16), ok)   # not pinned
    with pytest.raises(ValueError):
        pipe.submit(ok, torch.empty(8, 512, dtype=torch.bfloat16).pin_memory())
    with pytest.raises(IndexError):
        pipe.submit(ok, ok, layer=3)
