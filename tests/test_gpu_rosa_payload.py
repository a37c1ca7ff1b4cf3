"""GPU: the fused payload gradient of the Rosa training path
(ksd8_rosa_payload_bwd) against the straight-through input gradient of
Int8Linear (ste_input_grad, pinned to the reference's linear.py:88-94 by the
golden tests) followed by the reduction of rosa.py:164's product."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("act,S", [(torch.float32, 256), (torch.bfloat16, 256),
                                   (torch.float32, 64), (torch.bfloat16, 320)])
def test_payload_grad_matches_ste_formula(act, S):
    from ksdraft_b200 import _lib
    from ksdraft_b200.kernels.linear import ste_input_grad
    from ksdraft_b200.kernels.quant import quantize_last_dim
    g = torch.Generator().manual_seed(3)
    M = 1000      # S % 128 != 0: the last group is zero-padded (quant.py:40-44)
    payload = 1.0 + 0.2 * torch.randn(S, generator=g)
    payload[5] = payload[9] = payload[min(100, S - 1)] = 3.0   # three tied at the group maximum
    payload[S - 60] = -payload[S - 50].abs() - 2.0  # a negative group maximum
    sign = torch.where(torch.rand(M, S, generator=g) > 0.5, 1.0, -1.0)
    o = (payload * sign).to(act).cuda()
    sign = sign.to(act).cuda()
    oq, _ = quantize_last_dim(o)
    gx = torch.randn(M, S, generator=g).cuda() * 1e-2
    ref = (ste_input_grad(o.float(), oq, gx) * sign.float()).sum(0)
    parts = torch.empty(37, S, device="cuda")
    _lib.check(_lib.lib().ksd8_rosa_payload_bwd(
        o.data_ptr(), oq.data_ptr(), gx.data_ptr(), sign.data_ptr(), _lib.dtype_code(o), M, S,
        parts.data_ptr(), 37, None, _lib.stream_ptr(o.device)), "rosa_payload_bwd")
    got = parts.sum(0)
    rel = ((got - ref).norm() / ref.norm()).item()
    assert rel < 1e-5, rel
