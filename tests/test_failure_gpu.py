"""GPU: failure detection without a GPU fault.

The tensor-core indexer bounds every wait on its mbarrier pipeline.  A test
hook (DSA_TEST_INDEXER_STALL) makes its producer issue no loads, so every
wait runs out after 20 ms: the kernel must return (no hang), report
DSA_ERR_TIMEOUT through dsa_device_status, and leave the context usable."""
import pytest
import torch

import dsa_oracle as o

pytestmark = pytest.mark.gpu


def test_indexer_wait_timeout_is_reported_and_recoverable(cuda, monkeypatch):
    import _native
    from lightning_indexer import indexer_scores
    qi, ki, wi, *_ = (x.to(cuda) for x in o.make_inputs(1, 512, 4, 64, 1, 16, 16, dtype=torch.bfloat16))
    assert _native.device_status() == _native.DSA_OK
    monkeypatch.setenv("DSA_TEST_INDEXER_STALL", "1")
    indexer_scores(qi, ki, wi)                       # returns; the kernel gives up after 20 ms
    assert _native.device_status() == _native.DSA_ERR_TIMEOUT
    assert _native.device_status() == _native.DSA_OK  # the flag was cleared
    monkeypatch.delenv("DSA_TEST_INDEXER_STALL")
    out = indexer_scores(qi, ki, wi).cpu()           # the context still works
    assert _native.device_status() == _native.DSA_OK
    ref = o.indexer_scores(qi.cpu(), ki.cpu(), wi.cpu())
    fin = torch.isfinite(ref)
    assert torch.equal(torch.isfinite(out), fin)
    assert bool(((out[fin] - ref[fin]).abs() <= 2e-2 * ref[fin].abs() + 1e-2).all())
