"""Prompt-lookup speculative decoding, host side (CPU): the library's
n550_lookup_draft against the restatement of the reference's lookup_draft
(main_baremetal.c:567-584) in oracle/, on random histories over small
vocabularies (many matches) and the edge cases; and the oracle's restatement
of the speculative loop (main_baremetal.c:636-690) run on the reference's own
QWEN3_SPECULATIVE build (oracle/_ref/libref_spec.so) against the reference's
plain greedy run (tests/golden/greedy_ref.npz): the same tokens, as the
reference's design promises."""
import numpy as np
import pytest

import oracle
import n550_qwen3_bringup_handover_b200 as n5
from tests.conftest import GOLDEN


@pytest.mark.parametrize("vocab,ngram", [(3, 3), (5, 2), (8, 3), (50, 1), (4, 6)])
def test_lookup_draft_matches_reference_rule(vocab, ngram):
    rng = np.random.default_rng(vocab * 10 + ngram)
    for trial in range(300):
        n = int(rng.integers(0, 60))
        hist = rng.integers(0, vocab, n).astype(np.int32)
        max_k = int(rng.integers(0, 12))
        got = list(n5.lookup_draft(hist, ngram, max_k))
        want = oracle.lookup_draft(list(hist), ngram, max_k)
        assert got == want, (trial, list(hist), ngram, max_k)


def test_lookup_draft_edges():
    assert list(n5.lookup_draft([], 3, 5)) == []
    assert list(n5.lookup_draft([1, 2, 3], 3, 5)) == []                # no room for a match
    assert list(n5.lookup_draft([1, 2, 3, 4], 3, 5)) == []             # no repeat
    assert list(n5.lookup_draft([7, 7, 7, 7], 3, 5)) == [7]            # newest match
    assert list(n5.lookup_draft([1, 2, 9, 1, 2, 8, 1, 2], 2, 3)) == [8, 1, 2]
    assert list(n5.lookup_draft([1, 2, 9, 1, 2], 2, 0)) == []
    L = n5.lib()
    assert L.n550_lookup_draft(None, 5, 3, None, 2) == n5.ERR_ARG
    assert L.n550_lookup_draft(None, 0, 0, None, 2) == n5.ERR_ARG


@pytest.mark.skipif(not oracle.ref_available("spec"), reason="oracle/_ref not built")
def test_reference_speculative_loop_reproduces_greedy():
    """The reference's all-row-logits build under the restated loop emits the
    reference's greedy tokens (its scalar GEMM computes every row alike)."""
    z = np.load(GOLDEN / "greedy_ref.npz")
    prompt = z["prompt"]
    ref = oracle.RefModel(oracle.qw3m_blob(0, 0.02), "spec")
    toks, rounds, drafted, accepted = oracle.speculative_generate(ref, prompt, 20, 127)
    assert toks == list(z["scalar_tokens"][:20])
    assert rounds + accepted == 20
    assert drafted >= accepted
