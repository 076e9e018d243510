"""The speculative loop's host logic on the CPU: the prompt-lookup drafter
(lookup_draft, smollm_chat.rs:2982-3015) and the verify bookkeeping of
smollm_chat.rs:4205-4340 against a fake model whose greedy token is a fixed
function of the token prefix (so plain greedy decoding is known exactly)."""
import numpy as np
import torch

from spindle_b200.spec import LOOKUP_CORPUS_MAX, LookupCorpus, speculative_generate


def test_lookup_longest_ngram_most_recent():
    c = LookupCorpus()
    #         0  1  2  3  4  5  6  7  8  9 10 11 12 13
    c.remember([5, 1, 2, 3, 9, 8, 1, 2, 3, 7, 6, 4, 1, 2, 3])
    # suffix (1, 2, 3): the most recent earlier occurrence is at 6..8, followed by 7, 6, 4, 1
    d, ng = c.draft(4)
    assert (d, ng) == ([7, 6, 4, 1], 3)
    # k limits the draft; the end of the corpus limits it too
    assert c.draft(2) == ([7, 6], 3)
    assert c.draft(0) == ([], 0)


def test_lookup_two_gram_proposes_at_most_two():
    c = LookupCorpus()
    c.remember([4, 5, 6, 7, 8, 4, 5])
    assert c.draft(8) == ([6, 7], 2)


def test_lookup_four_gram_first_and_no_match():
    c = LookupCorpus()
    c.remember([1, 2, 3, 4, 10, 11, 9, 2, 3, 4, 20, 1, 2, 3, 4])
    # the 4-gram (1,2,3,4) at 0..3 wins over the later 3-gram (2,3,4) at 7..9
    assert c.draft(3) == ([10, 11, 9], 4)
    c2 = LookupCorpus()
    c2.remember([1, 2, 3, 4, 5])
    assert c2.draft(4) == ([], 0)


def test_lookup_stops_at_stop_token():
    c = LookupCorpus(stop_ids=[99])
    c.remember([1, 2, 3, 7, 99, 8, 1, 2, 3])
    assert c.draft(4) == ([7], 3)
    c = LookupCorpus(stop_ids=[7])
    c.remember([1, 2, 3, 7, 99, 8, 1, 2, 3])
    # the first candidate's draft is empty: the search goes on to shorter n-grams
    assert c.draft(4) == ([], 0)


def test_corpus_drops_oldest_half():
    c = LookupCorpus()
    c.remember(range(LOOKUP_CORPUS_MAX))
    assert len(c.tokens) == LOOKUP_CORPUS_MAX
    c.remember([1])
    assert len(c.tokens) == LOOKUP_CORPUS_MAX // 2
    assert c.tokens[-1] == 1 and c.tokens[0] == LOOKUP_CORPUS_MAX + 1 - LOOKUP_CORPUS_MAX // 2


class FakeDecoder:
    """Greedy token at a position = a hash of the tokens at positions 0..p
    (the "KV cache" is the position -> token map, rewritten by later passes)."""

    def __init__(self, vocab=50, period=None):
        self.cfg = {"n_layers": 2}
        self.kv = {}
        self.vocab = vocab
        self.period = period

    def _next(self, p):
        h = 1469598103934665603
        lo = 0 if self.period is None else max(0, p - self.period)
        for q in range(lo, p + 1):
            h = ((h ^ self.kv[q]) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
        return int(h % self.vocab)

    def forward_batch_range(self, pos0, l0, l1, tokens=None, hidden=None, n_max=64, stream=None, head=True):
        for i, t in enumerate(tokens):
            self.kv[pos0 + i] = int(t)
        return (None,)

    def forward_batch(self, tokens, pos0, logits=True, n_max=64, stream=None):
        for i, t in enumerate(tokens):
            self.kv[pos0 + i] = int(t)
        return None, torch.tensor([self._next(pos0 + i) for i in range(len(tokens))])

    def plain(self, prompt, n):
        self.kv = {}
        ctx = list(prompt)
        out = []
        for p, t in enumerate(ctx):
            self.kv[p] = t
        tok = self._next(len(ctx) - 1)
        for _ in range(n):
            out.append(tok)
            self.kv[len(ctx)] = tok
            ctx.append(tok)
            tok = self._next(len(ctx) - 1)
        return out


def test_loop_matches_plain_greedy_with_any_drafter():
    rng = np.random.default_rng(0)
    for period in [None, 3, 5]:   # short periods make the output repeat, so lookup drafts hit
        dec = FakeDecoder(vocab=7 if period else 50, period=period)
        prompt = rng.integers(0, dec.vocab, 40).tolist()
        want = dec.plain(prompt, 60)
        for drafter in [None,
                        lambda ctx, k: want[len(ctx) - len(prompt):][:k],                    # always right
                        lambda ctx, k: [(t + 1) % dec.vocab for t in want[len(ctx) - len(prompt):][:k]],  # always wrong
                        lambda ctx, k: want[len(ctx) - len(prompt):][:k // 2] + [0] * (k - k // 2)]:
            dec.kv = {}
            st = {}
            got = speculative_generate(dec, prompt, 60, drafter=drafter, stats=st, chunk=16)
            assert got == want, (period, st)
    # a fully right drafter needs far fewer passes than tokens
    dec = FakeDecoder()
    prompt = [1, 2, 3]
    want = dec.plain(prompt, 50)
    dec.kv = {}
    st = {}
    assert speculative_generate(dec, prompt, 50, drafter=lambda ctx, k: want[len(ctx) - 3:][:k], stats=st) == want
    assert st["passes"] <= 8 and st["accepted"] >= 40
