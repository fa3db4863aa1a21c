"""voom_moe_layer_noalloc: the MoE layer entry point that allocates nothing.

Callers that cannot allocate device memory (a runtime that owns the whole GPU
through its own pool, a serving loop that must not touch the allocator
between decode steps, a foreign host that only has the C ABI) use this
variant: its scratch is one fixed device array inside the library.  The test
calls it twice in a row through the C ABI and checks each result against the
allocating entry point (voom_moe_layer, caller-provided scratch) on the same
inputs, within the tolerance the MoE tests use (rel-L2 1e-2; the kernels are
the same, so the results are in fact identical).  It also checks that a call
beyond the stated limits is refused before anything is launched.  This file
is collected last so that a run stopping at its first failure has run every
other test already.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import moe as om

pytestmark = pytest.mark.gpu
TOL = 1e-2
VOOM_E_CAPACITY = -3


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.fixture(scope="module")
def layer(built_lib):
    from voom_b200.runtime import moe

    E, H, I = 16, 512, 256
    g = torch.Generator().manual_seed(77)
    ex = [tuple((torch.randn(s, generator=g) * 0.02).to(torch.bfloat16) for s in ((I, H), (I, H), (H, I)))
          for _ in range(E)]
    wr = torch.randn((E, H), generator=g).to(torch.bfloat16)
    nw = (1.0 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
    store = moe.ExpertStore([tuple(_bits(w) for w in e) for e in ex], "cuda:0")
    return moe.MoeLayer(store, wr.cuda(), nw.cuda(), top_k=4, norm_topk=True)


def _noalloc(layer, x: torch.Tensor, out: torch.Tensor, status: torch.Tensor) -> int:
    from voom_b200 import _device, _lib

    st = layer.store
    return _lib.load().voom_moe_layer_noalloc(
        st.table.data_ptr(), len(st), layer.router_w.data_ptr(), layer.norm_w.data_ptr(), layer.eps,
        x.data_ptr(), out.data_ptr(), int(x.shape[0]), st.H, st.I, layer.top_k, int(layer.norm_topk),
        st.gate_tiles, st.down_tiles, 1, status.data_ptr(), _device.stream_ptr(st.device, None))


def test_noalloc_matches_allocating_entry_point_twice(layer):
    g = torch.Generator().manual_seed(5)
    for T in (3, 8):  # two calls in a row, different inputs and sizes
        x = torch.randn((T, 512), generator=g).to(torch.bfloat16).cuda()
        want = layer(x)
        got = torch.empty_like(x)
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        assert _noalloc(layer, x, got, status) == 0
        torch.cuda.synchronize()
        assert int(status.item()) == 0 and int(layer.status.item()) == 0
        assert om.rel_l2(got.cpu(), want.cpu()) < TOL
        assert torch.equal(got, want)


def test_noalloc_refuses_sizes_beyond_its_limit(layer):
    x = torch.zeros((65, 512), dtype=torch.bfloat16, device="cuda")  # T > 64
    out = torch.empty_like(x)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert _noalloc(layer, x, out, status) == VOOM_E_CAPACITY
