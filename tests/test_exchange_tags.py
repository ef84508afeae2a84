"""The exchange-tag rule of the expert kernel, checked on the CPU.

Exchange words carry a 32-bit tag ``seq * 4096 + instance + 1`` (``mk_expert.cu``: launch sequence
number ``seq``, layer instance ``s * L + l``). The tag repeats every 2^20 launches, so a word that
no launch rewrote for that long could pass for fresh. The kernel closes this by having every launch
set to tag 0, at its exit, each word it did not write (``clear_stale_words``): rows >= T,
action-state words >= action_dim and parities the launch never uses; each CTA clears only words it
alone produces.

This model restates the ownership the kernel uses (column pairs split over the CTAs with
``part_lo``, the down partials' four groups, attention units ``u = head + 12 row`` on CTA u % G,
action-state row n on CTA n) and checks, for several geometries, that the words a launch writes and
the words it clears are disjoint and together cover every word of every exchange buffer, and that
each cleared word has exactly one clearing CTA. Tag 0 is never a valid tag.
"""
import itertools

import pytest

H, NH, TP, XWORDS, NGRP = 768, 12, 16, 32, 4
HWORDS, QKVWORDS = H // 2, 3 * H // 2
TAG_PERIOD = 1 << 20


def tag(seq, inst):
    return (seq * 4096 + inst + 1) & 0xFFFFFFFF


def part_lo(i, P, G):
    return (i * P) // G


def word_pos(kp):
    return (kp & ~7) | ((kp & 3) << 1) | ((kp >> 2) & 1)


def cta_split(i, G, I):
    lo, hi = part_lo(i, QKVWORDS, G), part_lo(i + 1, QKVWORDS, G)
    r = dict(qkv=(lo, hi - lo))
    lo, hi = part_lo(i, HWORDS, G), part_lo(i + 1, HWORDS, G)
    r["h"] = (lo, hi - lo)
    lo, hi = part_lo(i, I // 2, G), part_lo(i + 1, I // 2, G)
    r["gu"] = (lo, hi - lo)
    j = 0
    while j + 1 < NGRP and i >= part_lo(j + 1, G, NGRP):
        j += 1
    g0, gn = part_lo(j, G, NGRP), part_lo(j + 1, G, NGRP) - part_lo(j, G, NGRP)
    lo, hi = part_lo(i - g0, H // 2, gn), part_lo(i - g0 + 1, H // 2, gn)
    r["dp"] = (j * H + 2 * lo, 2 * (hi - lo))
    return r


def plan(G, I, T, n_steps, L, adim):
    """(written, cleared) as sets of (buffer, parity, row, word); cleared counts clearing CTAs."""
    n_inst = n_steps * L
    par_used = {0} | ({1} if n_inst >= 2 else set())
    xpar = {(s * L + L - 1) & 1 for s in range(n_steps - 1)}
    rw = dict(qkv=QKVWORDS, h2=HWORDS, qca=HWORDS, h3=HWORDS, hout=HWORDS, g=I // 2, dp=NGRP * H,
              y=HWORDS, yca=HWORDS, x=XWORDS)
    written = set()
    for b in rw:
        if b == "x":
            written |= {(b, p, n, a) for p in xpar for n in range(T) for a in range(adim)}
        else:
            written |= {(b, p, n, w) for p in par_used for n in range(T) for w in range(rw[b])}
    cleared = {}

    def clear(key):
        cleared[key] = cleared.get(key, 0) + 1
    for i in range(G):
        sp = cta_split(i, G, I)
        owned = [("qkv", *sp["qkv"], True), ("h2", *sp["h"], True), ("qca", *sp["h"], True), ("h3", *sp["h"], True),
                 ("hout", *sp["h"], True), ("g", *sp["gu"], True), ("dp", *sp["dp"], False)]
        for b, w0, nw, perm in owned:
            for p in (0, 1):
                r0 = T if p in par_used else 0
                for n in range(r0, TP):
                    for j in range(nw):
                        clear((b, p, n, word_pos(w0 + j) if perm else w0 + j))
        for u in range(i, NH * TP, G):
            n, h = u // NH, u % NH
            for p in (0, 1):
                if n < T and p in par_used:
                    continue
                for b in ("y", "yca"):
                    for k in range(32):
                        clear((b, p, n, h * 32 + k))
        if i < TP:
            for p, a in itertools.product((0, 1), range(XWORDS)):
                if not (p in xpar and i < T and a < adim):
                    clear(("x", p, i, a))
    allw = {(b, p, n, w) for b in rw for p in (0, 1) for n in range(TP) for w in range(rw[b])}
    return written, cleared, allw


def test_tags_repeat_after_two_to_the_twenty_launches_and_are_never_zero():
    for seq in (1, 2, 1000, TAG_PERIOD - 1, TAG_PERIOD, 3 * TAG_PERIOD + 5):
        for inst in (0, 1, 89, 4094):
            assert tag(seq, inst) != 0
            assert tag(seq + TAG_PERIOD, inst) == tag(seq, inst)
            assert tag(seq + 1, inst) != tag(seq, inst)


@pytest.mark.parametrize("G,I,T,n_steps,L,adim", [
    (148, 3072, 10, 9, 10, 7), (148, 3072, 16, 9, 10, 8), (148, 3072, 1, 1, 1, 1), (148, 1024, 5, 3, 2, 6),
    (132, 3072, 9, 2, 3, 3), (100, 1024, 16, 1, 2, 8), (148, 1024, 10, 2, 1, 7)])
def test_each_launch_writes_or_clears_every_exchange_word_once(G, I, T, n_steps, L, adim):
    written, cleared, allw = plan(G, I, T, n_steps, L, adim)
    assert not (written & set(cleared)), "a launch must not clear a word it writes"
    assert written | set(cleared) == allw, "every word is either written or cleared"
    assert max(cleared.values(), default=1) == 1, "one clearing CTA per word"
