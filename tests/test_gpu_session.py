"""The reference's session layer (ios/App/XJGlue.c, the C API its Swift app calls: xjg_host_new ->
xjg_host_chat -> xjg_host_reset) with CUDA stages, against the same code with the reference's CPU stages
(oracle/_ref/libxjglue_{cuda,cpu}.so, both built unmodified from XJGlue.c and core/ by oracle/Makefile):
the same streamed answers, turn after turn, greedy, and with the MTP head drafting tokens (speculative
decoding must not change the answer). On the reference's own tiny model, which carries a tokenizer."""
from __future__ import annotations

import pytest

from oracle import glue

pytestmark = pytest.mark.gpu

TURNS = ["hello", "tell me more", "and then?"]


def converse(which, path, mtp=None, draft=0):
    h = glue.Host(which, path, 512, mtp, draft)
    out = []
    try:
        for t in TURNS:
            ans, st = h.chat(t, 0.0, 24)
            out.append((ans, st.prompt_tokens, st.gen_tokens, st.n_past))
        h.reset()
        ans, st = h.chat(TURNS[0], 0.0, 24)
        out.append((ans, st.prompt_tokens, st.gen_tokens, st.n_past))
    finally:
        h.close()
    return out


@pytest.mark.skipif(not glue.available("cuda") or not glue.available("cpu"), reason="session-layer builds missing")
def test_session_chat_cuda_matches_cpu(tiny_path):
    want = converse("cpu", tiny_path)
    got = converse("cuda", tiny_path)
    assert got == want
    assert any(a for a, *_ in got)          # the model does answer


@pytest.mark.skipif(not glue.available("cuda") or not glue.available("cpu"), reason="session-layer builds missing")
def test_session_chat_with_mtp_drafts_matches_plain(tiny_path):
    want = converse("cpu", tiny_path)
    got = converse("cuda", tiny_path, tiny_path, 3)
    assert [g[0] for g in got] == [w[0] for w in want]
