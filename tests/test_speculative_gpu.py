"""All-row logits (n550_qwen3_forward_rows, the reference's QWEN3_SPECULATIVE
qwen3_forward_batch, qwen3.c:556-566) and prompt-lookup speculative
generation (n550_qwen3_generate_lookup, main_baremetal.c:636-690) on the GPU.

* Every row's logits of a call at 3, 12 and 40 tokens (the GEMV, the
  weight-streaming and the split-K routes) and of a following 5-token verify
  call, against the reference's own speculative build (oracle/_ref
  libref_spec.so, all-row logits) on the same weights: max |logit - ref| <=
  1e-2 of max |ref| per row, greedy choices equal or within that margin.
* Speculative generation gives the reference's greedy tokens
  (tests/golden/greedy_ref.npz, 64 tokens after the 32-token prompt), accepts
  drafts, and its rounds and draft counts equal the restated reference loop's.
"""
import numpy as np
import pytest

import oracle
import n550_qwen3_bringup_handover_b200 as n5
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-2


def rel(a, b):
    return float(np.abs(a.astype(np.float64) - b).max() / np.abs(b).max())


def same_choice(got, ref_logits):
    best = int(np.argmax(ref_logits))
    if got == best:
        return True
    return float(ref_logits[best] - ref_logits[got]) <= LOGIT_TOL * float(np.abs(ref_logits).max())


@pytest.fixture(scope="module")
def ref_spec():
    if not oracle.ref_available("spec"):
        pytest.skip("oracle/_ref not built")
    return oracle.RefModel(oracle.qw3m_blob(0, 0.02), "spec")


@pytest.mark.parametrize("n", [3, 12, 40])
def test_forward_rows_every_row_vs_reference(cuda, ref_spec, n):
    toks = oracle.synth_tokens(n + 5, 60 + n, 0x544F4B)
    m = n5.Model(seed=0, max_seqs=1, max_len=128, max_tokens=64)
    try:
        for t, p0 in ((toks[:n], 0), (toks[n:], n)):
            ids, lg = m.forward_rows(t, p0, want_logits=True)
            ref_spec.forward_batch(t, p0)
            rows = ref_spec.logits_rows()
            assert rows.shape[0] == len(t)
            for j in range(len(t)):
                assert rel(lg[j], rows[j]) <= LOGIT_TOL, (n, p0, j)
                assert same_choice(int(ids[j]), rows[j]), (n, p0, j)
                assert int(ids[j]) == int(np.argmax(lg[j]))
            ids_only, _ = m.forward_rows(t, p0)          # fused lm_head argmax path
            assert np.array_equal(ids_only, ids)
    finally:
        m.close()
    assert n5.device_status() == n5.OK


def test_generate_lookup_is_greedy_and_accepts_drafts(cuda, ref_spec):
    z = np.load(GOLDEN / "greedy_ref.npz")
    prompt, want = z["prompt"], [int(t) for t in z["scalar_tokens"]]
    m = n5.Model(seed=0, max_seqs=1, max_len=256, max_tokens=64)
    try:
        spec, st = m.generate_lookup(prompt, 64, max_draft=127)
        plain, st0 = m.generate_lookup(prompt, 64, max_draft=0)
    finally:
        m.close()
    assert n5.device_status() == n5.OK
    assert st0 == {"rounds": 64, "drafted": 0, "accepted": 0}
    for got in (list(spec), list(plain)):
        for i, (g, w) in enumerate(zip(got, want)):
            if g != w:     # only a near tie of the reference may part the sequences
                vals, ids = z["scalar_top_vals"][i], list(z["scalar_top_ids"][i])
                assert g in ids and vals[0] - vals[ids.index(g)] <= LOGIT_TOL * np.abs(vals).max()
                break
        else:
            assert len(got) == 64
    assert st["accepted"] > 0 and st["rounds"] + st["accepted"] == len(spec)
    if list(spec) == want:
        # same tokens: the same drafts, so the same rounds as the reference's loop
        toks, rounds, drafted, accepted = oracle.speculative_generate(ref_spec, prompt, 24, 127)
        m = n5.Model(seed=0, max_seqs=1, max_len=256, max_tokens=64)
        try:
            got24, st24 = m.generate_lookup(prompt, 24, max_draft=127)
        finally:
            m.close()
        assert list(got24) == toks
        assert (st24["rounds"], st24["drafted"], st24["accepted"]) == (rounds, drafted, accepted)


def test_generate_lookup_stops_at_eos(cuda):
    """The stop tokens end generation before they are emitted, in plain and in
    speculative generation (main_baremetal.c:650-670: an accepted draft that
    is a stop token ends the round too): with the reference's 6th greedy token
    as the only stop token, both return the 5 tokens before it."""
    z = np.load(GOLDEN / "greedy_ref.npz")
    prompt, want = z["prompt"], [int(t) for t in z["scalar_tokens"]]
    stop = want[5]
    if stop in want[:5]:
        pytest.skip("the stop token occurs earlier in this run")
    m = n5.Model(seed=0, max_seqs=1, max_len=256, max_tokens=64)
    try:
        plain, _ = m.generate_lookup(prompt, 64, max_draft=0, eos=(stop,))
        spec, _ = m.generate_lookup(prompt, 64, max_draft=127, eos=(stop,))
        capped, st = m.generate_lookup(prompt, 3, max_draft=127)
    finally:
        m.close()
    assert list(plain) == want[:5] and list(spec) == want[:5]
    assert list(capped) == want[:3] and st["rounds"] + st["accepted"] == 3
