"""The device loop control of generate() (pesti_generate_advance) against
the oracle's restatement of transformer/model.rs:508-531, on planned token
sequences that reach every exit (stop token, max_tokens, max_seq_len), and
inside a decode loop fed by the sampler and the device draws."""
import numpy as np
import pytest

import oracle as O
import synth

pytestmark = pytest.mark.gpu

REASON = {1: "stop", 2: "max_tokens", 3: "max_seq_len"}


def _run(steps_tok, stop, max_tokens, max_seq_len):
    import torch
    import pesti_sampler as ps
    B, T = steps_tok.shape[1], steps_tok.shape[0]
    st = ps.DecodeState(B, max_tokens, max_seq_len, stop)
    for t in range(T):
        st.advance(torch.from_numpy(steps_tok[t].astype(np.int32)).cuda())
    torch.cuda.synchronize()
    return st


@pytest.mark.parametrize("max_tokens,max_seq_len", [(10, 8), (6, 100), (0, 5), (12, 1)])
def test_generate_advance_matches_the_loop(max_tokens, max_seq_len):
    rng = np.random.default_rng(max_tokens * 7 + max_seq_len)
    B, T = 40, 14
    steps = rng.integers(0, 16, size=(T, B)).astype(np.uint32)
    stop = [3, 11]
    st = _run(steps, stop, max_tokens, max_seq_len)
    seqs = st.sequences()
    done = st.done.cpu().numpy()
    last = st.last.cpu().numpy().view(np.uint32)
    running = 0
    for b in range(B):
        want, why = O.generate_control(list(map(int, steps[:, b])), stop, max_tokens, max_seq_len)
        assert seqs[b] == want, b
        assert REASON.get(int(done[b])) == why, (b, done[b], why)
        if want:
            assert int(last[b]) == want[-1]
        running += why is None
    assert st.active() == running


def test_decode_loop_on_the_device():
    """Ten steps of a batched decode loop with device draws: every step's
    tokens equal the sampler's own, and the loop control keeps them."""
    import torch
    import pesti_sampler as ps
    B, V, T = 8, 32000, 10
    s = ps.Sampler(0)
    rng = ps.DeviceRng(B, seed=5, first_stream=0)
    st = ps.DecodeState(B, max_tokens=T, max_seq_len=64, stop_tokens=[7])
    cfg = ps.SamplingConfig(0.8, 0.95, 40)
    toks = []
    for t in range(T):
        x = torch.from_numpy(synth.make_logits(1, B=B)[:, :V] * (1.0 + 0.1 * t)).cuda()
        u = rng.draw()
        tok = s.sample_batch(x, cfg, u)
        toks.append(tok.cpu().numpy().view(np.uint32).copy())
        st.advance(tok)
    torch.cuda.synchronize()
    steps = np.stack(toks)
    for b, seq in enumerate(st.sequences()):
        want, _ = O.generate_control(list(map(int, steps[:, b])), [7], T, 64)
        assert seq == want
