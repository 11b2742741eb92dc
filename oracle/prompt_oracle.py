"""CPU restatement of the reference's TTS prompt builder — TEST INFRASTRUCTURE ONLY.

Restates zonos2_build_prompt (src/zonos2-prompt.cpp:54-133) and the conditioning layout of
zonos2_hparams (src/zonos2.h:41-46) in plain Python, with the silence table written out in
the reference's own 17-row form (src/zonos2-prompt.cpp:19-37). Only tests/ use it, as the
checker of z2b_build_prompt; the product never imports it.
"""
from __future__ import annotations

RATE, QUALITY, BG, ACCURATE = 8, [12, 12, 12, 8, 8, 8], 2, 1
DEFAULT_QFEAT, DEFAULT_QBUCKET = 5, 3

_S0 = [568, 778, 338, 524, 967, 360, 728, 550, 90]
_S1 = [568, 778, 10, 674, 364, 981, 741, 378, 731]
_SM = [568, 804, 10, 674, 364, 981, 568, 378, 731]
_S16 = [568, 778, 721, 842, 264, 974, 989, 507, 308]
SILENCE = [_S0, _S1] + [list(_SM) for _ in range(14)] + [_S16]


def build_prompt(text: bytes, n_codebooks=9, text_vocab=519, audio_pad=1025, prepend_silence=True,
                 speaking_rate_bucket=-1, quality_buckets=None, add_speaker_slot=False,
                 clean_speaker_background=True, accurate_mode=True):
    """Rows [n][n_codebooks + 1] and spk_pos, as zonos2_build_prompt returns them."""
    ncb, tv, pad = n_codebooks, text_vocab, audio_pad
    sum_q = sum(QUALITY)
    base = tv - RATE - sum_q - BG - ACCURATE
    rows = []

    def pad_row(t):
        return [pad] * ncb + [t]

    spk_pos = -1
    if add_speaker_slot:
        rows.append(pad_row(tv))
        spk_pos = 0
        if BG > 0:
            rows.append(pad_row(base + RATE + sum_q + (0 if clean_speaker_background else 1)))
            if ACCURATE > 0 and accurate_mode:
                rows.append(pad_row(base + RATE + sum_q + BG))
    if speaking_rate_bucket >= 0:
        rows.append(pad_row(base + speaking_rate_bucket))
    qb = list(quality_buckets or [])
    if not qb:
        qb = [-1] * len(QUALITY)
        qb[DEFAULT_QFEAT] = DEFAULT_QBUCKET
    prefix = 0
    for f, cnt in enumerate(QUALITY):
        if f < len(qb) and qb[f] >= 0:
            rows.append(pad_row(base + RATE + prefix + qb[f]))
        prefix += cnt
    rows.append(pad_row(2))
    rows += [pad_row(192 + b) for b in text]
    rows.append(pad_row(3))
    if prepend_silence:
        for t in range(17):
            r = [pad] * (ncb + 1)
            for c in range(min(ncb, 9)):
                if t >= c:
                    r[c] = SILENCE[t - c][c]
            r[ncb] = tv
            rows.append(r)
    return rows, spk_pos
