"""CPU stand-in for one chunk pair of context-parallel attention (test
infrastructure for the ring's exchange logic on gloo ranks): exact fp32
attention of a query chunk against one key chunk, merged into (out, lse) by
the log-sum-exp rule the kernel's partial form uses."""

import torch


def cpu_partial(q, k, v, causal, scale, out, lse, accumulate):
    s = torch.matmul(q.float(), k.float().transpose(-1, -2)) * scale
    if causal:
        L = s.shape[-1]
        s = s.masked_fill(torch.ones(L, L, dtype=torch.bool).triu(1), float("-inf"))
    lse_new = torch.logsumexp(s, dim=-1)
    o_new = torch.matmul(torch.softmax(s, dim=-1), v.float())
    if not accumulate:
        out.copy_(o_new.to(out.dtype))
        lse.copy_(lse_new)
        return
    m = torch.maximum(lse, lse_new)
    w_old = torch.exp(lse - m)
    w_new = torch.exp(lse_new - m)
    tot = w_old + w_new
    merged = (out.float() * (w_old / tot)[..., None] + o_new * (w_new / tot)[..., None])
    out.copy_(merged.to(out.dtype))
    lse.copy_(m + torch.log(tot))
