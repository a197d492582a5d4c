"""GraphedStep: a GMLP forward + backward captured once in a CUDA graph and replayed on new
inputs gives the same bits as the eager step on those inputs."""
import pytest

pytestmark = pytest.mark.gpu


def test_graphed_gmlp_step_matches_eager(cuda):
    import torch
    from macrogpt_jax_b200 import _capi as C
    from macrogpt_jax_b200.einsum import Einsum, Rngs, scaled_normal_init
    from macrogpt_jax_b200.graphs import GraphedStep
    from macrogpt_jax_b200.mlp import GMLP
    d, h, T = 256, 512, 512
    mlp = GMLP.override(fused_proj=Einsum.override(initializer=scaled_normal_init(d ** -0.5)),
                        down_proj=Einsum.override(initializer=scaled_normal_init(h ** -0.5)))(
        model_d=d, hidden_d=h, rngs=Rngs(3))
    assert mlp.fused()
    params = list(mlp.parameters())

    def step(xb, dyb):
        xl = xb.detach().requires_grad_(True)
        y = mlp(xl)
        y.backward(dyb)
        out = (y.detach(), xl.grad, *[p.grad for p in params])
        for p in params:
            p.grad = None
        return out

    gen = torch.Generator(device=cuda)
    gen.manual_seed(4)
    inputs = [(torch.randn((2, T // 2, d), generator=gen, device=cuda).to(torch.bfloat16),
               (torch.randn((2, T // 2, d), generator=gen, device=cuda) * 1e-3).to(torch.bfloat16))
              for _ in range(3)]
    graphed = GraphedStep(step, *inputs[0])
    for xb, dyb in inputs[1:] + inputs[:1]:
        want = [t.clone() for t in step(xb, dyb)]
        got = graphed(xb, dyb)
        torch.cuda.synchronize()
        assert len(got) == len(want)
        for g, w in zip(got, want):
            assert torch.equal(g, w)
    assert C.device_status() == 0
