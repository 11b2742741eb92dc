"""Teacher-forced quality evaluation (zonos2.cpp_b200/quality.py) against a literal restatement
of the reference tool's loops (src/perplexity.cpp:130-375): perplexity, the KL base file's
byte layout (read and written in the reference's version-2 format), and the KL battery
(quantiles, top-1 agreement, log-probability differences). A seeded stand-in model supplies the
logits on the CPU; the GPU test scores the tiny model against itself through z2b_logits."""
from __future__ import annotations

import math
import struct

import numpy as np
import pytest

NCB, AV, PAD = 3, 11, 10


class _Hp:
    n_codebooks, audio_vocab, audio_pad_id, spk_dim = NCB, AV, PAD, 4


class _FakeModel:
    """Logits seeded by the sequence's content (and speaker), plus a perturbation scale."""

    def __init__(self, noise=0.0):
        self.hp = _Hp()
        self.noise = noise

    def logits(self, ids, spk=None, spk_pos=0, spk_emotion_delta=None):
        ids = np.asarray(ids, np.int32)
        key = int(ids.sum()) + (0 if spk is None else int(1000 * float(np.sum(spk))) + 7 * spk_pos)
        g = np.random.default_rng(key)
        x = g.standard_normal((len(ids), NCB, AV)).astype(np.float32) * 3
        if self.noise:
            x = x + np.random.default_rng(key + 1).standard_normal(x.shape).astype(np.float32) * self.noise
        return x


def _seqs():
    import z2b.quality as Q
    g = np.random.default_rng(0)
    out = []
    for n in (7, 12, 2):
        ids = g.integers(0, AV, (n, NCB + 1)).astype(np.int32)
        ids[g.random((n, NCB + 1)) < 0.2] = PAD                # padded labels to skip
        out.append(Q.Sequence(ids))
    out.append(Q.Sequence(g.integers(0, 10, (9, NCB + 1)).astype(np.int32), spk=np.ones(4, np.float32), spk_pos=1))
    return out


def _ref_log_softmax(row):
    mx = row[0]
    for v in row[1:]:
        if v > mx:
            mx = v
    se = sum(math.exp(float(np.float32(v - mx))) for v in row)
    lse = np.float32(mx + np.float32(math.log(se)))
    return [np.float32(v - lse) for v in row]


def _ref_events(model, s):
    lg = model.logits(s.ids, s.spk, s.spk_pos if s.spk_pos >= 0 else 0)
    out = []
    for t in range(len(s.ids) - 1):
        for cb in range(NCB):
            L = int(round(float(s.ids[t + 1][cb])))
            if L == PAD or L < 0 or L >= AV:
                continue
            out.append((_ref_log_softmax(lg[t, cb]), L, cb))
    return out


def test_perplexity_matches_reference_loops():
    import z2b.quality as Q
    m, seqs = _FakeModel(), _seqs()
    got = Q.perplexity(m, seqs)
    nll, cnt = [0.0] * NCB, [0] * NCB
    for s in seqs:
        for lp, L, cb in _ref_events(m, s):
            nll[cb] += -float(lp[L])
            cnt[cb] += 1
    tot = sum(cnt)
    assert got["events"] == tot
    assert abs(got["ppl"] - math.exp(sum(nll) / tot)) < 1e-9 * got["ppl"]
    for c in range(NCB):
        assert abs(got["ppl_per_codebook"][c] - math.exp(nll[c] / cnt[c])) < 1e-6


def test_base_layout_and_self_divergence(tmp_path):
    import z2b.quality as Q
    m, seqs = _FakeModel(), _seqs()
    path = str(tmp_path / "base.bin")
    Q.kl_base(m, seqs, path)
    b = open(path, "rb").read()
    # the reference writer's order: magic, version, ncb, av, pad, n_seq, per-seq meta, ids (+spk), events
    assert b[:8] == b"Z2KLDIV2" and struct.unpack_from("<5I", b, 8) == (2, NCB, AV, PAD, len(seqs))
    off = 28
    for s in seqs:
        assert struct.unpack_from("<IiI", b, off) == (len(s.ids), s.spk_pos if s.spk is not None else -1,
                                                       0 if s.spk is None else len(s.spk))
        off += 12
    for s in seqs:
        assert np.array_equal(np.frombuffer(b, np.float32, s.ids.size, off), s.ids.ravel().astype(np.float32))
        off += 4 * s.ids.size
        if s.spk is not None:
            off += 4 * len(s.spk)
    ev = [e for s in seqs for e in _ref_events(m, s)]
    lp = np.frombuffer(b, np.float32, len(ev) * AV, off).reshape(-1, AV)
    assert off + lp.nbytes == len(b)
    assert np.abs(lp - np.array([e[0] for e in ev], np.float32)).max() <= 1e-6
    r = Q.kl_divergence(m, path)
    assert r["kld_max"] == 0.0 and r["top1_agreement"] == 1.0 and r["ppl_ratio"] == 1.0


def test_divergence_matches_reference_loops(tmp_path):
    import z2b.quality as Q
    ref_m, test_m, seqs = _FakeModel(), _FakeModel(noise=0.7), _seqs()
    path = str(tmp_path / "base.bin")
    Q.kl_base(ref_m, seqs, path)
    got = Q.kl_divergence(test_m, path)
    kl, agree, dl, rn, tn = [], 0, [], 0.0, 0.0
    for s in seqs:
        for (lr, L, cb), (lt, _, _) in zip(_ref_events(ref_m, s), _ref_events(test_m, s)):
            k = sum(math.exp(float(a)) * float(np.float32(a - b)) for a, b in zip(lr, lt))
            kl.append(max(k, 0.0))
            agree += int(np.argmax(lr) == np.argmax(lt))
            dl.append(float(lt[L]) - float(lr[L]))
            rn += -float(lr[L])
            tn += -float(lt[L])
    n = len(kl)
    kl.sort()
    assert got["events"] == n
    assert abs(got["kld_mean"] - sum(kl) / n) < 1e-6
    for key, q in (("kld_median", 0.5), ("kld_p90", 0.9), ("kld_p99", 0.99)):
        assert abs(got[key] - kl[int(round(q * (n - 1)))]) < 1e-6
    assert got["top1_agreement"] == agree / n
    assert abs(got["dlogp_mean"] - sum(dl) / n) < 1e-9
    assert abs(got["ppl_ratio"] - math.exp(tn / n) / math.exp(rn / n)) < 1e-9


def test_base_errors(tmp_path):
    import z2b.quality as Q
    p = tmp_path / "bad.bin"
    p.write_bytes(b"NOTABASE" + b"\0" * 40)
    with pytest.raises(ValueError):
        Q.read_base(str(p))
    p.write_bytes(b"Z2KLDIV2" + struct.pack("<5I", 1, NCB, AV, PAD, 0))
    with pytest.raises(ValueError):
        Q.read_base(str(p))


@pytest.mark.gpu
def test_gpu_self_divergence_is_zero(model_dir, tmp_path):
    """The tiny model scored against its own base through z2b_logits: deterministic logits give
    KLD 0 and full agreement; its perplexity is finite and equals the base's."""
    import z2b.quality as Q
    import z2b.runtime as R
    import z2b.synth as S
    from tests.util import prompt
    m = R.Model(S.cached("tiny", directory=model_dir))
    seqs = [Q.Sequence(prompt(24, 1)), Q.Sequence(prompt(17, 2)),
            Q.Sequence(prompt(20, 3), spk=np.random.default_rng(3).standard_normal(m.hp.spk_dim).astype(np.float32),
                       spk_pos=2)]
    path = str(tmp_path / "base.bin")
    base = Q.kl_base(m, seqs, path)
    r = Q.kl_divergence(m, path)
    p = Q.perplexity(m, seqs)
    assert r["kld_max"] == 0.0 and r["top1_agreement"] == 1.0
    assert math.isfinite(p["ppl"]) and abs(p["ppl"] - base["ppl_ref"]) < 1e-9 * p["ppl"]
    m.close()
