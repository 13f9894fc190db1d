"""The synthetic stack's batch invariance: decoding b sequences together or
one at a time gives bit-identical route ids and tokens.  This is the
property that makes the route journal identical across GPU counts (an
expert-parallel rank decodes b/N of the sequences)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from dee_b200 import build
    build.build()
    return torch


def test_stack_decode_is_batch_invariant(torch_cuda, tmp_path):
    torch = torch_cuda
    from dee_b200.journal import verify_chain
    from dee_b200.stack import StackSpec, SyntheticStack, journal_bytes, seed_tokens
    spec = StackSpec(layers=3, experts=16, hidden=512, inter=512, topk=6, vocab=1024, seed=7)
    B, steps = 4, 3
    first = torch.from_numpy(seed_tokens(spec, B)).cuda()

    def run(tokens, first_t):
        st = SyntheticStack(torch, spec, tokens=tokens)
        ids = torch.empty((steps, spec.layers, tokens, spec.topk), dtype=torch.int32, device="cuda")
        tok = torch.empty((steps, tokens), dtype=torch.int32, device="cuda")
        st.decode(first_t, steps, ids, tok)
        torch.cuda.synchronize()
        assert st.engine.sync_status() == 0 and st.router.sync_status() == 0
        return ids.cpu().numpy(), tok.cpu().numpy()

    ids_b, tok_b = run(B, first)
    for i in range(B):
        ids_1, tok_1 = run(1, first[i:i + 1].contiguous())
        assert np.array_equal(ids_1[:, :, 0], ids_b[:, :, i])
        assert np.array_equal(tok_1[:, 0], tok_b[:, i])
    # the decode moves: tokens change and experts vary across layers
    assert len(np.unique(tok_b)) > 1
    j = journal_bytes(ids_b, run_id="test")
    assert j.count(b"\n") == steps * spec.layers
    p = tmp_path / "routed_experts.jsonl"
    p.write_bytes(j)
    n, _ = verify_chain(p)
    assert n == steps * spec.layers
