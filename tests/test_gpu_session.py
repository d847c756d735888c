"""The reference's session layer (ios/App/XJGlue.c, the C API its Swift app calls: xjg_host_new ->
xjg_host_chat -> xjg_host_reset) with CUDA stages, against the same code with the reference's CPU stages
(oracle/_ref/libxjglue_{cuda,cpu}.so, both built unmodified from XJGlue.c and core/ by oracle/Makefile):
the same streamed answers, turn after turn, greedy, and with the MTP head drafting tokens (speculative
decoding must not change the answer); and the two-machine split over the reference's TCP protocol
(core/xj_net.c) with a CUDA worker serving a CPU host and a CPU worker serving a CUDA host (layers
[2, 5) on the worker). On the reference's own tiny model, which carries a tokenizer."""
from __future__ import annotations

import pytest

from oracle import glue

pytestmark = pytest.mark.gpu

TURNS = ["hello", "tell me more", "and then?"]


def converse(which, path, mtp=None, draft=0, **remote):
    h = glue.Host(which, path, 512, mtp, draft, **remote)
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


def free_port():
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not glue.available("cuda") or not glue.available("cpu"), reason="session-layer builds missing")
@pytest.mark.parametrize("worker_backend,host_backend", [("cuda", "cpu"), ("cpu", "cuda")])
def test_worker_interop_over_tcp(tiny_path, worker_backend, host_backend):
    want = converse("cpu", tiny_path)
    port, pin = free_port(), 4242
    w = glue.Worker(worker_backend, tiny_path, 2, 5, port, pin)
    try:
        import time
        time.sleep(0.5)                          # the worker starts listening
        got = converse(host_backend, tiny_path, worker="127.0.0.1", port=port, pin=pin, s1=2, s2=5)
    finally:
        w.close()
    assert [g[0] for g in got] == [x[0] for x in want]
