"""The device decoder (wc_decoder_*, decoder.cu) against the CPU restatement
of internal/decoder (oracle/whistle_oracle.c) on a synthetic Whistle-shaped
decoder: 8 layers of width 512 in 4 mHC lanes, int8 self- and
cross-attention, engram at layers 3 and 7, the tied CQ4 head.

- The int8 cross-attention memory (cross.go:181 project) is the oracle's
  bit for bit: codes and scales.
- Every Extend step's logits (decoder.go:252) match the oracle's: bit for
  bit on almost every value, and all within DECODER_RTOL of the largest
  |logit| of the row. The one allowed source of difference is a float64
  sum's order (the norms' sums of squares run as a tree on the device):
  it can move a float32 result by one ulp when the float64 value lies
  within about 2^-44 of a float32 rounding boundary, and libm's and CUDA's
  double exp can differ likewise.
- GreedyMemory (greedy.go:40) gives the oracle's language and text tokens,
  EOS flags and counts for every stream: identical token ids.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# Tolerance on a logit against the oracle's, relative to the row's largest
# |logit| (the north star's 1e-5 relative for fp32 outputs).
DECODER_RTOL = 1e-5

LANGS_SMALL = [8 + i for i in range(7)]


@pytest.fixture(scope="module")
def model(wb, orc):
    w = wb.synth.DecoderWeights(seed=4200, vocab=16384)
    return w, orc.OracleDecoder(w)


def _enc(wb, cuda, streams, frames, seed):
    enc = wb.synth.encoder_output(np.random.default_rng(seed), streams, frames)
    return enc, cuda.from_numpy(enc).cuda()


@pytest.mark.parametrize("flags", [0, 2], ids=["graph", "eager"])
def test_memory_bit_exact(wb, orc, cuda, model, flags):
    w, od = model
    S, F = 3, 64
    enc, denc = _enc(wb, cuda, S, F, 11)
    dec = wb.decoder.Decoder(w, max_streams=4, max_frames=F, max_positions=16, flags=flags)
    dec.Memory(denc)
    cuda.cuda.synchronize()
    xh, xq, xv = w.x_heads, w.x_qk, w.x_vd
    for l in (0, 3, 7):
        k8p, ksp, v8p, vsp = dec.memory_of(l)
        k8 = _dev_array(cuda, k8p, S * F * xh * xq, np.int8)
        ks = _dev_array(cuda, ksp, S * F * xh, np.float32)
        v8 = _dev_array(cuda, v8p, S * F * xh * xv, np.int8)
        vs = _dev_array(cuda, vsp, S * F * xh, np.float32)
        for b in range(S):
            st = od.state(8, F)
            st.memory(enc[b])
            ok8, oks, ov8, ovs = st.memory_of(l)
            n8, nsc = F * xh * xq, F * xh
            assert np.array_equal(k8[b * n8:(b + 1) * n8], ok8), (l, b)
            assert np.array_equal(ks[b * nsc:(b + 1) * nsc].view(np.uint32), oks.view(np.uint32)), (l, b)
            nv = F * xh * xv
            assert np.array_equal(v8[b * nv:(b + 1) * nv], ov8), (l, b)
            assert np.array_equal(vs[b * nsc:(b + 1) * nsc].view(np.uint32), ovs.view(np.uint32)), (l, b)


def _dev_array(cuda, ptr, n, dtype):
    """A host copy of n elements of device memory at ptr."""
    from cuda.bindings import runtime as cudart

    out = np.empty(n, dtype)
    cuda.cuda.synchronize()
    (err,) = cudart.cudaMemcpy(out.ctypes.data, ptr, out.nbytes, cudart.cudaMemcpyKind.cudaMemcpyDeviceToHost)
    assert err == cudart.cudaError_t.cudaSuccess
    return out


@pytest.mark.parametrize("flags", [0, 2], ids=["graph", "eager"])
def test_extend_logits_match_oracle(wb, orc, cuda, model, flags):
    w, od = model
    S, F, steps = 3, 48, 10
    enc, denc = _enc(wb, cuda, S, F, 12)
    dec = wb.decoder.Decoder(w, max_streams=S, max_frames=F, max_positions=steps + 2, flags=flags)
    dec.Memory(denc)
    states = []
    for b in range(S):
        st = od.state(steps + 2, F)
        st.memory(enc[b])
        states.append(st)
    rng = np.random.default_rng(5)
    logits = cuda.empty((S, w.vocab), dtype=cuda.float32, device="cuda")
    nxt = cuda.empty(S, dtype=cuda.int32, device="cuda")
    exact = total = 0
    for step in range(steps):
        toks = rng.integers(0, w.vocab, size=S).astype(np.int32)
        dec.Extend(cuda.from_numpy(toks).cuda(), logits, nxt)
        got = logits.cpu().numpy()
        got_next = nxt.cpu().numpy()
        for b in range(S):
            want = states[b].extend(int(toks[b]))
            assert np.all(np.isfinite(got[b]))
            err = np.abs(got[b] - want).max() / np.abs(want).max()
            assert err <= DECODER_RTOL, (step, b, err)
            exact += int(np.sum(got[b].view(np.uint32) == want.view(np.uint32)))
            total += want.size
            assert got_next[b] == int(np.argmax(want)), (step, b)
    assert dec.Len() == steps
    # Bit-exact on (nearly) every logit: the only differences allowed are
    # the rare float64-order and exp last-bit cases.
    assert exact >= 0.99 * total, f"{exact} of {total} logits bit-exact"


def test_greedy_tokens_identical(wb, orc, cuda, model):
    w, od = model
    S, F, max_tok = 32, 375, 32
    S_ = wb.synth
    enc, denc = _enc(wb, cuda, S, F, 13)
    dec = wb.decoder.Decoder(w, max_streams=S, max_frames=F, max_positions=max_tok + 1)
    dec.Memory(denc)
    tokens, counts, lang, eos = dec.GreedyMemory(S_.WHISTLE_BOS, S_.WHISTLE_LANGS, S_.WHISTLE_EOS, max_tok)
    tokens, counts, lang, eos = (t.cpu().numpy() for t in (tokens, counts, lang, eos))
    otok, ocnt, olang, oeos = od.greedy_streams(enc, S_.WHISTLE_BOS, S_.WHISTLE_LANGS, S_.WHISTLE_EOS, max_tok,
                                                threads=8)
    assert np.array_equal(lang, olang)
    assert np.array_equal(counts, ocnt)
    assert np.array_equal(eos, oeos)
    assert np.array_equal(tokens, otok[:, :max_tok - 1])
    # Not a degenerate run: the streams do not all say the same thing.
    assert len({tuple(t) for t in otok}) > 1


def test_greedy_twice_restarts(wb, orc, cuda, model):
    """A second Memory on the same decoder starts every stream afresh: the
    greedy run repeats bit for bit (the captured step graph is reused)."""
    w, od = model
    S, F = 4, 32
    S_ = wb.synth
    enc, denc = _enc(wb, cuda, S, F, 14)
    dec = wb.decoder.Decoder(w, max_streams=S, max_frames=F, max_positions=12)
    runs = []
    for _ in range(2):
        dec.Memory(denc)
        runs.append([t.cpu().numpy() for t in dec.GreedyMemory(S_.WHISTLE_BOS, LANGS_SMALL, S_.WHISTLE_EOS, 10)])
    for a, b in zip(*runs):
        assert np.array_equal(a, b)


def test_decoder_errors(wb, cuda, model):
    w, _ = model
    S_ = wb.synth
    with pytest.raises(wb.Panic, match="room for"):
        wb.decoder.Decoder(w, max_streams=0)
    dec = wb.decoder.Decoder(w, max_streams=2, max_frames=16, max_positions=4)
    with pytest.raises(wb.Panic, match="no memory"):
        dec.GreedyMemory(S_.WHISTLE_BOS, LANGS_SMALL, S_.WHISTLE_EOS, 3)
    _, denc = _enc(wb, cuda, 2, 16, 15)
    with pytest.raises(wb.Panic, match="encoder output"):
        dec.Memory(cuda.zeros((3, 16, 512), dtype=cuda.float32, device="cuda"))
    dec.Memory(denc)
    with pytest.raises(wb.Panic, match="positions exceed"):
        dec.GreedyMemory(S_.WHISTLE_BOS, LANGS_SMALL, S_.WHISTLE_EOS, 9)
    with pytest.raises(wb.Panic, match="out of range"):
        dec.GreedyMemory(w.vocab, LANGS_SMALL, S_.WHISTLE_EOS, 3)
