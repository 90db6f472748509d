"""Two layers stepped on two unordered CUDA streams give exactly the results of
the same steps run one after the other.

The fused up + down forward launch has blocks that wait for other blocks' up
tiles, so its whole grid must be resident and two such launches must not
overlap; the launcher orders a launch after the device's previous one when that
ran on another stream.  Without that ordering the launches would also share
their row-block counters.
"""

import pytest
import torch

from tests.test_layer_gpu import make_layer

pytestmark = pytest.mark.gpu


def _step(layer, x, g):
    xi = x.clone().requires_grad_(True)
    layer.zero_grad(set_to_none=True)
    out, _aux, _f = layer(xi)
    out.backward(g)
    return out.detach(), xi.grad, layer.w1.grad, layer.w2.grad


def test_layers_on_two_streams_match_sequential(device):
    from moe_b200.kernels import _ops

    H, sizes, k = 768, [(4, 512), (8, 256), (4, 128)], 2
    layers = [make_layer(H, sizes, k, seed=s, device=device) for s in (0, 1)]
    gen = torch.Generator(device="cpu").manual_seed(7)
    xs = [torch.randn(2, 2048, H, generator=gen).to(device, torch.bfloat16) for _ in range(2)]
    gs = [torch.randn(2, 2048, H, generator=gen).to(device, torch.bfloat16) for _ in range(2)]

    ref = [_step(layers[i], xs[i], gs[i]) for i in range(2)]
    torch.cuda.synchronize()

    streams = [torch.cuda.Stream(device=device) for _ in range(2)]
    for s in streams:
        s.wait_stream(torch.cuda.current_stream(device))
    got = [[], []]
    for _rep in range(3):
        for i in (0, 1):  # queued back to back, no ordering between the streams
            with torch.cuda.stream(streams[i]):
                got[i].append(_step(layers[i], xs[i], gs[i]))
    torch.cuda.synchronize()
    _ops.check_device_status(device)
    for i in (0, 1):
        for res in got[i]:
            for a, b in zip(res, ref[i]):
                assert torch.equal(a, b)
