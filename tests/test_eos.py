"""EOS / countdown / max_frames / next-row bookkeeping of a stream (z2b_slot_after_frame,
the per-frame logic of zonos2_slot_sample, src/zonos2-graph.cpp:843-870) against a
line-by-line Python restatement of the reference, on random frame sequences with
end-of-audio codes planted in chosen codebooks. Host only: no GPU."""
from __future__ import annotations

import numpy as np
import pytest

import z2b.runtime as R


def _hp(ncb=9, eoa=1024, text_vocab=519):
    hp = R.HParams()
    hp.n_codebooks, hp.eoa_id, hp.text_vocab, hp.audio_vocab = ncb, eoa, text_vocab, 1025
    return hp


def _reference(st, frame, eoa, ncb, text_vocab, max_frames, keep):
    """zonos2_slot_sample after sampling `frame` (src/zonos2-graph.cpp:852-868)."""
    frame_idx = st["step"]
    max_eoa = -1
    for cb in range(ncb):
        if frame[cb] == eoa:
            max_eoa = cb
    if st["eos_frame"] < 0 and max_eoa >= 0:
        st["eos_frame"] = max(0, frame_idx - max_eoa)
        st["countdown"] = ncb + 1
    finished = False
    if st["countdown"] > 0:
        st["countdown"] -= 1
        finished = st["countdown"] == 0
    st["next_ids"] = list(frame[:ncb]) + [text_vocab]
    st["step"] += 1
    if not keep or finished or st["step"] >= max_frames:
        st["done"] = True
    return keep


def _run(hp, frames, max_frames, stop_at=None):
    ref = dict(step=0, eos_frame=-1, countdown=-1, done=False, next_ids=[])
    s = R.Slot(index=3, n_past=17)
    out = []
    for i, f in enumerate(frames):
        keep = stop_at is None or i != stop_at
        kr = _reference(ref, [int(x) for x in f], hp.eoa_id, hp.n_codebooks, hp.text_vocab, max_frames, keep)
        kc = R.slot_after_sample(hp, s, f, max_frames, keep)
        assert kr == kc
        assert (s.step, s.eos_frame, s.countdown, s.done, s.next_ids) == \
            (ref["step"], ref["eos_frame"], ref["countdown"], ref["done"], ref["next_ids"]), i
        out.append((s.step, s.eos_frame, s.countdown, s.done))
        if s.done:
            break
    assert s.n_past == 17 and s.index == 3            # the caller advances n_past, not this call
    return out


@pytest.mark.parametrize("seed", range(20))
def test_eos_countdown_matches_reference(seed):
    hp = _hp()
    g = np.random.default_rng(seed)
    frames = g.integers(0, 1024, (60, hp.n_codebooks)).astype(np.int32)
    at = int(g.integers(0, 40))
    cbs = g.choice(hp.n_codebooks, int(g.integers(1, 4)), replace=False)
    frames[at, cbs] = hp.eoa_id                       # the codebook offset: eos_frame = step - last eoa codebook
    if seed % 3 == 0:
        frames[at + 2, 0] = hp.eoa_id                 # a later eoa does not restart the countdown
    trace = _run(hp, frames, max_frames=10 ** 9)
    step, eos, cd, done = trace[-1]
    assert done and cd == 0
    assert eos == max(0, at - int(cbs.max()))
    assert step == at + hp.n_codebooks + 1            # countdown of n_codebooks + 1 frames


def test_eos_in_the_first_frames_clamps_to_zero():
    hp = _hp()
    frames = np.zeros((20, hp.n_codebooks), np.int32)
    frames[1, 8] = hp.eoa_id
    assert _run(hp, frames, 10 ** 9)[-1][1] == 0      # max(0, 1 - 8)


def test_max_frames_and_stop_callback():
    hp = _hp()
    frames = np.ones((30, hp.n_codebooks), np.int32)
    trace = _run(hp, frames, max_frames=7)
    assert len(trace) == 7 and trace[-1][3]
    trace = _run(hp, frames, max_frames=100, stop_at=4)
    assert len(trace) == 5 and trace[-1][3]


def test_bad_arguments_are_rejected():
    hp = _hp(ncb=40)                                  # more columns than Z2B_MAX_ROW
    with pytest.raises(R.Z2BError):
        R.slot_after_sample(hp, R.Slot(index=0), np.zeros(40, np.int32), 10)
