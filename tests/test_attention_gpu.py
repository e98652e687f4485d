"""The paged grouped-query attention kernel (sc_paged_attention) of the synthetic decoder against a float32 torch
reference of the same softmax(q k^T / 16) v on the same bfloat16 inputs: windows of 1 to 5 and 8 new tokens (the
kernel's four-, two- and one-group forms), contexts that end inside a chunk, a page and a round of a group's pages,
the sequence's pages scattered through the cache."""

import math

import pytest
import torch

from strata_mlx_b200 import _lib
from strata_mlx_b200.decoder import HEAD_DIM, PAGE

pytestmark = pytest.mark.gpu


def reference(q, kseq, vseq, ctx):
    t, hq, d = q.shape
    hkv = kseq.shape[1]
    out = torch.empty((t, hq, d), dtype=torch.float32, device=q.device)
    for i in range(t):
        n = ctx - t + i + 1
        for h in range(hq):
            kv = h // (hq // hkv)
            s = (kseq[:n, kv].float() @ q[i, h].float()) / math.sqrt(d)
            out[i, h] = torch.softmax(s, 0) @ vseq[:n, kv].float()
    return out


@pytest.mark.parametrize("tokens", [1, 2, 3, 4, 5, 8])
@pytest.mark.parametrize("ctx", [5, 300, 1000, 4113, 20000])
def test_paged_attention_is_the_softmax_product(cuda, tokens, ctx):
    if ctx < tokens:
        pytest.skip("the window is part of the context")
    g = torch.Generator(device="cuda").manual_seed(ctx + tokens)
    hq, hkv = 16, 2
    max_tokens = ctx + 40
    pages = -(-max_tokens // PAGE)
    k = torch.randn((pages, PAGE, hkv, HEAD_DIM), generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn((pages, PAGE, hkv, HEAD_DIM), generator=g, device="cuda").to(torch.bfloat16)
    table = torch.randperm(pages, generator=torch.Generator().manual_seed(7)).to(torch.int32).cuda()
    q = torch.randn((tokens, hq, HEAD_DIM), generator=g, device="cuda").to(torch.bfloat16)
    ctx_dev = torch.tensor([ctx], dtype=torch.int32, device="cuda")
    lib = _lib.load()
    n = lib.sc_paged_attention_workspace(max_tokens, hkv)
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    out = torch.empty((tokens, hq, HEAD_DIM), dtype=torch.bfloat16, device="cuda")
    rc = lib.sc_paged_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), table.data_ptr(), ctx_dev.data_ptr(),
                                max_tokens, tokens, hq, hkv, HEAD_DIM, 1.0 / 16.0, out.data_ptr(), ws.data_ptr(), n,
                                torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    seq = table.long()
    kseq = k[seq].reshape(-1, hkv, HEAD_DIM)[:ctx]
    vseq = v[seq].reshape(-1, hkv, HEAD_DIM)[:ctx]
    want = reference(q, kseq, vseq, ctx)
    torch.cuda.synchronize()
    err = (out.float() - want).abs().max().item()
    # probabilities are rounded to bfloat16 for the value product, the output to bfloat16
    assert err <= 2e-2 * want.abs().max().item(), err
