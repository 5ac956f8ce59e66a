"""GPU: the host-buffer pipeline (HostChain) gives the same bits as the
device-resident chained pass, for both Q/K layouts and several chunk sizes,
over consecutive passes (the second pass refills the device slots of the
first while its copies out may still be draining)."""

import pytest
import torch

from hrm_layer_ops import chain, ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("token_major,chunk", [(True, 128), (True, 512), (False, None)])
def test_host_chain_matches_device_pass(cuda, token_major, chunk):
    g = torch.Generator(device=cuda).manual_seed(3)
    B, S, H, D, HID, I, V = 2, 512, 4, 128, 512, 768, 1000

    def rn(shape, std=1.0, mean=0.0):
        return (torch.randn(shape, generator=g, device=cuda) * std + mean).to(torch.bfloat16)

    w = chain.ChainWeights(table=rn((V, HID), 0.02), w1=rn(HID, 0.1, 1.0), w2=rn(HID, 0.1, 1.0),
                           rope=ops.rope_table(S, D), scale=22.6, eps=1e-5, theta=10000.0)
    T = B * S
    qk = (B, S, H, D) if token_major else (B, H, S, D)
    dev_in = dict(ids=torch.randint(0, V + 5, (T,), generator=g, device=cuda, dtype=torch.int32),
                  q=rn(qk), k=rn(qk), o=rn((T, HID)), gate=rn((T, I), 0.5), up=rn((T, I), 0.5))
    bf = dict(dtype=torch.bfloat16, device=cuda)
    want = dict(q=dev_in["q"].clone(), k=dev_in["k"].clone(), h=torch.empty((T, HID), **bf),
                n1=torch.empty((T, HID), **bf), r=torch.empty((T, HID), **bf), n2=torch.empty((T, HID), **bf),
                y=torch.empty((T, I), **bf))
    chain.run_device(w, dev_in["ids"], want["q"], want["k"], dev_in["o"], dev_in["gate"], dev_in["up"], want["h"],
                     want["n1"], want["r"], want["n2"], want["y"], 0, token_major=token_major)
    torch.cuda.synchronize()

    hc = chain.HostChain(w, B, H, S, D, HID, I, chunk_tokens=chunk, token_major=token_major, device=cuda)
    host_in = {n: t.cpu().pin_memory() for n, t in dev_in.items()}
    outs = []
    for _ in range(2):  # two back-to-back passes, no host synchronisation between them
        host_out = {n: torch.zeros(t.shape, dtype=t.dtype).pin_memory() for n, t in want.items()}
        hc.run(host_in, host_out)
        outs.append(host_out)
    torch.cuda.synchronize()
    for host_out in outs:
        for n, t in want.items():
            assert torch.equal(host_out[n].view(torch.int16), t.cpu().view(torch.int16)), n
