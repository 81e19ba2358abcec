"""Host-buffer calls of >= 4096 tokens are pipelined in chunks of whole routing blocks (copies on
their own streams, overlapping the compute). Chunking must not change the result: with the
deterministic down path the output is bitwise the same as one unchunked device-buffer call, and
with the default atomic path it agrees to fp32 summation order (GPU).
"""
import numpy as np
import pytest
import torch

import diffuse_moe as dm
import synth
from test_gpu_parity import rel_l2


@pytest.mark.gpu
@pytest.mark.slow
def test_chunked_host_call_matches_device_call(monkeypatch):
    spec = synth.config("c2")  # S shape, q8_0
    L = dm.MoELayer(spec.hparams(), synth.make_layer(spec))
    n = 6144  # five chunks of 24 to 64 routing blocks
    x = synth.make_input(n, spec.H, 13)
    xd = torch.from_numpy(x).cuda()
    dev_det = L.forward(xd, deterministic=True)
    torch.cuda.synchronize()
    host_det = L.forward(x, deterministic=True)  # numpy in: host mode, chunked
    assert np.array_equal(host_det.view(np.uint32), dev_det.cpu().numpy().view(np.uint32))
    host = L.forward(x)
    assert rel_l2(host, dev_det.cpu().numpy()) < 1e-6
    # equal chunks forced by DMOE_HOST_CHUNK (three of 2048 tokens): bitwise the same again
    monkeypatch.setenv("DMOE_HOST_CHUNK", "2048")
    eq_det = L.forward(x, deterministic=True)
    assert np.array_equal(eq_det.view(np.uint32), host_det.view(np.uint32))
    monkeypatch.delenv("DMOE_HOST_CHUNK")
    # a call that is not a whole number of routing blocks is never chunked (block routing off)
    x2 = synth.make_input(n - 7, spec.H, 14)
    a = L.forward(x2)
    b = L.forward(torch.from_numpy(x2).cuda()).cpu().numpy()
    assert rel_l2(a, b) < 1e-6
    L.close()
