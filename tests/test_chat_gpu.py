"""Text in, text out on the GPU runtime (n550_qwen3_chat): the reference's
chat mode (main.c:137-185) with the reference's own tokenizer and forward
(oracle/_ref: tokenizer.c on tok.bin, qwen3.c + kernels_scalar.c) as the
checker. The prompt ids must be identical, the generated ids the reference's
greedy ids (or a near tie of the reference, within the fast-mode logit
tolerance, after which the runs part), and the reply text the reference
tokenizer's decoding of the ids; plain and speculative generation agree."""
import numpy as np
import pytest

import oracle
import n550_qwen3_bringup_handover_b200 as n5

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-2
EOS = (151645, 151643)


@pytest.mark.skipif(not oracle.tokenizer_available() or not oracle.ref_available("scalar"),
                    reason="oracle/_ref not built")
def test_chat_turn_vs_reference(cuda):
    prompt = "你好，请介绍一下你自己"
    tok = n5.Tokenizer(oracle.TOK_PATH)
    rtok = oracle.RefTokenizer()
    full = ("<|im_start|>user\n" + prompt + "<|im_end|>\n<|im_start|>assistant\n"
            "<think>\n\n</think>\n\n").encode()
    ref_in = rtok.encode(full)
    assert np.array_equal(tok.chat(prompt), ref_in)

    m = n5.Model(seed=0, max_seqs=1, max_len=256, max_tokens=128)
    try:
        text, ids = m.chat(tok, prompt, max_new=16)
        text_s, ids_s = m.chat(tok, prompt, max_new=16, max_draft=127)
    finally:
        m.close()
    assert n5.device_status() == n5.OK

    # the reference's chat loop: prefill, then one token at a time
    ref = oracle.RefModel(oracle.qw3m_blob(0, 0.02), "scalar")
    logits = ref.forward_batch(ref_in, 0)
    want, steps = [], []
    for i in range(16):
        nxt = oracle.argmax(logits)
        if nxt in EOS:
            break
        want.append(nxt)
        steps.append(logits)
        logits = ref.forward_batch(np.array([nxt], np.int32), len(ref_in) + i)
    for got in (list(ids), list(ids_s)):
        for i, (g, w) in enumerate(zip(got, want)):
            if g != w:
                lg = steps[i]
                assert lg[w] - lg[g] <= LOGIT_TOL * np.abs(lg).max(), (i, g, w)
                break
        else:
            assert len(got) == len(want)
    assert text == rtok.decode(ids) and text_s == rtok.decode(ids_s)
    if list(ids) == want:
        assert list(ids_s) == want
