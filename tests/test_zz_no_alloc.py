"""ufp8_amax_quant_noalloc (scratch in static device arrays) against ufp8_amax_quant (caller's
amax buffer): quantized bytes and inverse scale bit-identical, for two calls in a row with
different tensors (the second must not see the first one's scratch), both formats, aligned and
unaligned inputs, ragged and empty tensors.  Kept in its own file, collected last."""
import pytest

pytestmark = pytest.mark.gpu


def _pair(x, fmt):
    import torch
    from macrogpt_jax_b200 import _capi as C
    n = x.numel()
    stream = torch.cuda.current_stream().cuda_stream
    q_ref = torch.empty(n, dtype=torch.uint8, device=x.device)
    amax_ref = torch.empty(1, dtype=torch.float32, device=x.device)
    inv_ref = torch.empty(1, dtype=torch.float32, device=x.device)
    C.amax_quant(x.data_ptr(), n, fmt, q_ref.data_ptr(), amax_ref.data_ptr(), inv_ref.data_ptr(), stream)
    q = torch.empty(n, dtype=torch.uint8, device=x.device)
    inv = torch.full((1,), -1.0, dtype=torch.float32, device=x.device)
    C.amax_quant_noalloc(x.data_ptr(), n, fmt, q.data_ptr(), inv.data_ptr(), stream)
    torch.cuda.synchronize()
    return q, inv, q_ref, inv_ref


@pytest.mark.parametrize("fmt", [0, 1], ids=["e4m3", "e5m2"])
@pytest.mark.parametrize("n_a,n_b", [(1 << 20, 3 * 65536 + 7), (200_003, 65536), (1, 0)])
def test_two_calls_match_amax_quant(cuda, fmt, n_a, n_b):
    import torch
    gen = torch.Generator(device=cuda)
    gen.manual_seed(11)
    a = (torch.randn(n_a, generator=gen, device=cuda) * 30.0).to(torch.bfloat16)
    b = (torch.randn(max(n_b, 1), generator=gen, device=cuda) * 0.01).to(torch.bfloat16)[:n_b]
    for x in (a, b):  # the second, smaller-amax tensor must not inherit the first's maximum
        q, inv, q_ref, inv_ref = _pair(x, fmt)
        assert torch.equal(q, q_ref)
        assert torch.equal(inv.view(torch.int32), inv_ref.view(torch.int32))


def test_unaligned_and_special_values(cuda):
    import torch
    base = torch.randn(300_001, device=cuda).to(torch.bfloat16)
    base[12345] = float("inf")
    x = base[1:]  # 2-byte aligned, not 16-byte aligned: scalar paths
    for fmt in (0, 1):
        q, inv, q_ref, inv_ref = _pair(x, fmt)
        assert torch.equal(q, q_ref)
        assert torch.equal(inv.view(torch.int32), inv_ref.view(torch.int32))


def test_oversize_is_rejected_without_launch(cuda):
    import torch
    from macrogpt_jax_b200 import _capi as C
    x = torch.zeros(16, dtype=torch.bfloat16, device=cuda)
    q = torch.empty(16, dtype=torch.uint8, device=cuda)
    inv = torch.empty(1, dtype=torch.float32, device=cuda)
    with pytest.raises(C.UFP8Error, match="exceed the static scratch"):
        C.amax_quant_noalloc(x.data_ptr(), 4096 * 65536 + 1, 0, q.data_ptr(), inv.data_ptr(),
                             torch.cuda.current_stream().cuda_stream)
    assert C.device_status() == 0
