"""Speculative decoding at temperature 0 on the batch forward: the prompt-lookup
drafter and the verify loop of the reference (smollm_chat.rs:2973-3015 and
:4205-4340; docs/speculative_decoding.md).

Each verify pass runs the pending token plus the draft through one
`sg_forward_batch` (every position's greedy token in one call), keeps the
longest prefix of drafts equal to the model's own greedy tokens and takes the
model's token at the first mismatch (or the extra one after a full accept).
The token stream is therefore exactly plain greedy decoding's; rejected
positions' K/V rows lie past the accepted position and are rewritten by the
next pass.
"""
LOOKUP_CORPUS_MAX = 16 * 1024   # smollm_chat.rs:29
LOOKUP_MAX_NGRAM = 4            # :31
LOOKUP_MIN_NGRAM = 2            # :32


class LookupCorpus:
    """The prompt-lookup corpus: every token fed or generated, the oldest half
    dropped when it passes LOOKUP_CORPUS_MAX (remember_tokens, :2973-2980)."""

    def __init__(self, stop_ids=()):
        self.tokens = []
        self.stop_ids = set(stop_ids)

    def remember(self, ids):
        self.tokens.extend(int(t) for t in ids)
        if len(self.tokens) > LOOKUP_CORPUS_MAX:
            del self.tokens[:len(self.tokens) - LOOKUP_CORPUS_MAX // 2]

    def draft(self, k):
        """lookup_draft (:2982-3015): the most recent earlier occurrence of the
        corpus's last n tokens, longest n first (4 down to 2), proposes the up
        to k tokens that followed it (at most 2 for a 2-gram), cut at a stop
        token.  Returns (draft, n) with n = 0 when nothing matched."""
        c, n = self.tokens, len(self.tokens)
        if k == 0:
            return [], 0
        for ng in range(LOOKUP_MAX_NGRAM, LOOKUP_MIN_NGRAM - 1, -1):
            if n <= ng:
                continue
            pat = c[n - ng:]
            for i in range(n - ng - 1, -1, -1):   # starts that end before the suffix itself
                if c[i + ng - 1] == pat[-1] and c[i:i + ng] == pat:
                    s = i + ng
                    kk = min(k, 2) if ng == LOOKUP_MIN_NGRAM else k
                    d = []
                    for t in c[s:min(s + kk, n)]:
                        if t in self.stop_ids:
                            break
                        d.append(t)
                    if d:
                        return d, ng
        return [], 0


def speculative_generate(dec, prompt, n_new, draft_len=8, drafter=None, stop_ids=(), chunk=64, stats=None):
    """Greedy decoding of n_new tokens after `prompt` with speculative verify
    passes (the loop of smollm_chat.rs:4205-4340 at temperature 0).

    dec: a spindle_b200.decoder.Decoder.  drafter(context, k) -> list of at
    most k proposed tokens (default: prompt lookup over the context, with the
    reference's backoff after a rejected 2-gram draft and its draft length
    that grows by 2 after a full accept).  Returns the n_new tokens, identical
    to dec.generate(prompt, n_new).  stats (a dict, optional) receives
    passes, drafted, accepted and single steps."""
    prompt = [int(t) for t in prompt]
    # the prompt (feed): every position's K/V rows, then the first token from the last
    n_max = max(chunk, draft_len + 1)
    for c0 in range(0, len(prompt) - 1, chunk):
        part = prompt[c0:min(c0 + chunk, len(prompt) - 1)]
        dec.forward_batch_range(c0, 0, dec.cfg["n_layers"], tokens=part, n_max=n_max, head=False)
    _, g = dec.forward_batch([prompt[-1]], len(prompt) - 1, logits=False, n_max=n_max)
    return speculative_decode(dec, int(g[0].item()), len(prompt), n_new, prompt, draft_len, drafter, stop_ids,
                              n_max, stats)


def speculative_decode(dec, tok, pos, n_new, context, draft_len=8, drafter=None, stop_ids=(), n_max=64, stats=None):
    """The verify loop from a fed context: `tok` is the greedy token after
    `context` (not yet in the KV caches), `pos` its position.  Returns the
    n_new tokens from tok on, identical to plain greedy decoding."""
    prompt = [int(t) for t in context]
    corpus = LookupCorpus(stop_ids)
    corpus.remember(prompt)
    use_lookup = drafter is None
    st = {"passes": 0, "drafted": 0, "accepted": 0, "steps": 0} if stats is None else stats
    for key in ("passes", "drafted", "accepted", "steps"):
        st.setdefault(key, 0)
    n_max = max(n_max, draft_len + 1)
    out = []
    backoff = skip = 0
    k_dyn = draft_len
    while len(out) < n_new:
        if tok in corpus.stop_ids:
            break
        out.append(tok)
        corpus.remember([tok])
        if len(out) >= n_new:
            break
        k = min(k_dyn, max(n_new - len(out) - 1, 0))   # room for the token the pass adds
        draft = []
        if k > 0:
            if use_lookup:
                d, ng = corpus.draft(k)
                if skip == 0 or ng > LOOKUP_MIN_NGRAM:
                    draft = d
            else:
                draft = [int(t) for t in drafter(prompt + out, k)][:k]
        skip = max(skip - 1, 0)
        if not draft:
            _, g = dec.forward_batch([tok], pos, logits=False, n_max=n_max)
            pos += 1
            tok = int(g[0].item())
            st["steps"] += 1
            continue
        batch = [tok] + draft
        _, g = dec.forward_batch(batch, pos, logits=False, n_max=n_max)
        greedy = g.tolist()
        st["passes"] += 1
        st["drafted"] += len(draft)
        # position i's greedy token predicts batch[i + 1] = draft[i]
        accepted = 0
        correction = None
        for i, d_tok in enumerate(draft):
            if greedy[i] != d_tok:
                correction = greedy[i]
                break
            accepted += 1
            out.append(d_tok)
            corpus.remember([d_tok])
            if len(out) >= n_new:
                break
        st["accepted"] += accepted
        pos += 1 + accepted
        if len(out) >= n_new:
            break
        if accepted == 0:
            backoff = min(max(backoff * 2, 1), 16)
            skip = backoff
        else:
            backoff = 0
        k_dyn = max(min(k_dyn + 2, 7), draft_len) if accepted == len(draft) else draft_len
        tok = correction if correction is not None else greedy[len(draft)]
    return out[:n_new]
