"""Test infrastructure: a CPU restatement of internal/search's beam search
(search/beam.go, options.go) over the oracle decoder's states, the checker
for the device search (wc_decoder_beam). Never part of the product.

The expander seam is the reference's (beam.go:68): ``expand(hs, n,
allowed)`` returns each hypothesis' n best candidates, so the reference's
hand-computed step and pick tests run against this restatement with their
own scripted expanders, and ``Stepper`` runs it on ``OracleDecoder``
states, forking a state that another hypothesis still holds (beam.go:537
own, decoder.go:223 State.Fork).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

NORM_NONE, NORM_LEN, NORM_POW, NORM_GNMT = 1, 2, 3, 4
LEN_TEXT, LEN_TEXT_EOS, LEN_SEQ = 1, 2, 3
STOP_ALL, STOP_BEST, STOP_K, STOP_HF = 1, 2, 3, 4
ADMIT_TOPK, ADMIT_ABOVE_LIVE = 1, 2
LANG_ARGMAX, LANG_ARGMAX_SCORED, LANG_BEAM = 1, 2, 3


class OptionsError(ValueError):
    pass


@dataclass
class Options:
    """options.go:105 Options (no Adjust hook, Whisper's finished rule)."""

    beams: int = 5
    max_tokens: int = 0
    language: int = -1  # index into the language list, -1 to detect
    norm: int = NORM_LEN
    alpha: float = 1.0
    length: int = LEN_TEXT
    stop: int = STOP_K
    admit: int = ADMIT_ABOVE_LIVE
    lang: int = LANG_ARGMAX

    def validate(self) -> None:
        """options.go:160 Validate."""
        bad = "search: invalid options"
        if self.beams < 1:
            raise OptionsError(f"{bad}: {self.beams} beams")
        if self.max_tokens < 0:
            raise OptionsError(f"{bad}: max tokens {self.max_tokens}")
        if not NORM_NONE <= self.norm <= NORM_GNMT:
            raise OptionsError(f"{bad}: norm {self.norm}")
        if not LEN_TEXT <= self.length <= LEN_SEQ:
            raise OptionsError(f"{bad}: length {self.length}")
        if not STOP_ALL <= self.stop <= STOP_HF:
            raise OptionsError(f"{bad}: stop {self.stop}")
        if not ADMIT_TOPK <= self.admit <= ADMIT_ABOVE_LIVE:
            raise OptionsError(f"{bad}: admit {self.admit}")
        if not LANG_ARGMAX <= self.lang <= LANG_BEAM:
            raise OptionsError(f"{bad}: language step {self.lang}")
        if math.isnan(self.alpha) or math.isinf(self.alpha):
            raise OptionsError(f"{bad}: alpha {self.alpha}")

    def penalty(self, l: int) -> float:
        """options.go:213 penalty."""
        if self.norm == NORM_LEN:
            return float(max(l, 1))
        if self.norm == NORM_POW:
            return math.pow(float(max(l, 1)), self.alpha)
        if self.norm == NORM_GNMT:
            return math.pow((5 + float(l)) / 6, self.alpha)
        return 1.0


@dataclass
class Cand:
    tok: int
    lp: float
    adj: float


@dataclass
class Hyp:
    """beam.go:38 hyp."""

    seq: list
    text: int
    lps: list = field(default_factory=list)
    lang_lp: float = 0.0
    sum: float = 0.0
    adj: float = 0.0
    eos: bool = False
    st: object = None
    fed: int = 0

    def text_len(self) -> int:
        return max(0, len(self.seq) - self.text)

    def text_tokens(self) -> list:
        return [] if len(self.seq) < self.text else self.seq[self.text:]


def log_softmax(v) -> np.ndarray:
    """beam.go:605 logSoftmax in float64, the sum in index order."""
    x = np.asarray(v, np.float32).astype(np.float64)
    m = float(np.max(x))
    s = float(np.cumsum(np.exp(x - m))[-1])
    return x - (m + math.log(s))


def candidates(lp, n: int, allowed=None) -> list:
    """beam.go:559 candidates (no adjust): the n best by log p, best first,
    ties to the lower id; allowed restricts them (ties to the earlier)."""
    lp = np.asarray(lp, np.float64)
    if allowed is not None:
        order = sorted(range(len(allowed)), key=lambda i: -lp[allowed[i]])
        return [Cand(int(allowed[i]), float(lp[allowed[i]]), float(lp[allowed[i]])) for i in order[:n]]
    order = np.argsort(-lp, kind="stable")[:n]
    return [Cand(int(t), float(lp[t]), float(lp[t])) for t in order]


class Beam:
    """beam.go:188 beam: the bookkeeping between steps."""

    def __init__(self, opt: Options, eos: int):
        self.opt, self.eos, self.fin = opt, eos, []

    def length(self, h: Hyp) -> int:
        l = h.text_len()
        if self.opt.length == LEN_SEQ:
            l = len(h.seq)
        if h.eos and self.opt.length != LEN_TEXT:
            l += 1
        return l

    def score(self, h: Hyp) -> float:
        return h.adj / self.opt.penalty(self.length(h))

    def final(self, h: Hyp) -> float:
        return self.score(h)

    def child(self, h: Hyp, c: Cand) -> Hyp:
        k = Hyp(seq=h.seq, text=h.text, lps=h.lps + [c.lp], lang_lp=h.lang_lp, sum=h.sum + c.lp, adj=h.adj + c.adj,
                st=h.st, fed=h.fed)
        if c.tok == self.eos:
            k.eos = True
        else:
            k.seq = h.seq + [c.tok]
        return k

    def kids(self, ex, alive: list) -> list:
        k = self.opt.beams
        cs = ex.expand(alive, k + 1, None)
        kids = []
        for i, h in enumerate(alive):
            for j, c in enumerate(cs[i]):
                if j > k and c.tok == self.eos:
                    continue
                kids.append(self.child(h, c))
        kids.sort(key=lambda h: -h.adj)  # stable: ties keep the parent's rank, then the candidate's
        return kids

    def step(self, ex, alive: list):
        """beam.go:247 step: the next live hypotheses and whether done."""
        k = self.opt.beams
        kids = self.kids(ex, alive)
        if self.opt.stop == STOP_ALL:
            pool = self.fin + kids
            pool.sort(key=lambda h: -self.score(h))
            self.fin, alive = [], []
            for h in pool[:k]:
                (self.fin if h.eos else alive).append(h)
            return alive, len(alive) == 0
        alive = []
        for rank, h in enumerate(kids):
            if not h.eos:
                alive.append(h)
                if len(alive) == k:
                    break
                continue
            if self.opt.admit == ADMIT_TOPK and rank >= k:
                continue
            self.finish(h)
        return alive, self.done(alive)

    def worst(self) -> int:
        w = 0
        for i, f in enumerate(self.fin):
            if self.score(f) < self.score(self.fin[w]):
                w = i
        return w

    def finish(self, h: Hyp) -> None:
        k = self.opt.beams
        if self.opt.stop == STOP_K:
            if len(self.fin) < k:
                self.fin.append(h)
        elif self.opt.stop == STOP_HF:
            self.fin.append(h)
            if len(self.fin) > k:
                del self.fin[self.worst()]
        else:
            self.fin.append(h)

    def done(self, alive: list) -> bool:
        if not alive:
            return True
        if not self.fin:
            return False
        live = max(self.score(h) for h in alive)
        if self.opt.stop == STOP_K:
            return len(self.fin) >= self.opt.beams
        if self.opt.stop == STOP_BEST:
            return max(self.score(h) for h in self.fin) >= live
        if self.opt.stop == STOP_HF:
            if len(self.fin) < self.opt.beams:
                return False
            return min(self.score(h) for h in self.fin) >= live
        return False

    def pick(self, alive: list, done: bool) -> Optional[Hyp]:
        """beam.go:113 pick."""
        pool = list(self.fin)
        if not done or not pool:
            live = alive
            if self.opt.stop == STOP_K:
                live = sorted(alive, key=lambda h: -h.adj)[:max(self.opt.beams - len(pool), 0)]
            pool = pool + list(live)
        best = None
        for h in pool:
            if best is None or self.final(h) > self.final(best):
                best = h
        return best


class Stepper:
    """beam.go:492 stepper over OracleState states."""

    def __init__(self, vocab: int):
        self.vocab = vocab

    def expand(self, hs: list, n: int, allowed) -> list:
        refs = {}
        for h in hs:
            refs[id(h.st)] = refs.get(id(h.st), 0) + 1
        for h in hs:  # own: a state another hypothesis holds is forked
            if refs[id(h.st)] > 1:
                refs[id(h.st)] -= 1
                h.st = h.st.fork()
                refs[id(h.st)] = 1
        out = []
        for h in hs:
            logits = None
            for tok in h.seq[h.fed:]:
                logits = h.st.extend(tok)
            h.fed = len(h.seq)
            out.append(candidates(log_softmax(logits), n, allowed))
        return out


@dataclass
class Result:
    tokens: list
    eos: bool
    lang: int
    lang_lp: float
    score: float
    logprobs: list


def search(state, bos: int, langs, eos: int, opt: Options, max_tokens: int) -> Result:
    """beam.go:73 Beam from an oracle state that holds a clip's memory."""
    opt.validate()
    ex = Stepper(None)
    ids = [langs[opt.language]] if opt.language >= 0 else list(langs)
    n = min(opt.beams, len(ids)) if opt.lang == LANG_BEAM else 1
    prompt = [bos]
    start = Hyp(seq=list(prompt), text=len(prompt) + 1, st=state)
    cs = ex.expand([start], n, ids)
    alive = []
    for c in cs[0]:
        h = Hyp(seq=prompt + [c.tok], text=start.text, lang_lp=c.lp, st=start.st, fed=start.fed)
        if opt.lang != LANG_ARGMAX and opt.language < 0:
            h.sum = h.adj = c.lp
        alive.append(h)
    s = Beam(opt, eos)
    done = False
    step = 0
    while step < max_tokens - 1 and not done:
        alive, done = s.step(ex, alive)
        step += 1
    best = s.pick(alive, done)
    return Result(tokens=best.text_tokens(), eos=best.eos, lang=best.seq[best.text - 1], lang_lp=best.lang_lp,
                  score=s.final(best), logprobs=list(best.lps))
