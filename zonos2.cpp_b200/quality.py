"""Teacher-forced quality evaluation: perplexity and KL divergence against a reference model.

Replaces the reference's zonos2-perplexity tool (src/perplexity.cpp:150-375) on this library's
teacher-forced logits (z2b_logits, the same kernels as the decode step). Each (frame t,
codebook c) pair with a real label is one prediction event: the logits after row t score row
t + 1's code in codebook c; labels equal to the audio pad id, or outside the audio vocabulary,
are skipped (the delay pattern's padding).

The KL workflow keeps one model in memory at a time, as the reference's does: ``kl_base``
writes the reference model's log-probabilities of every event to a base file, and
``kl_divergence`` scores another model (a quantisation) against it. The base file has the
reference tool's version-2 layout, so a base written by either tool is read by the other:
  "Z2KLDIV2", u32 version 2, u32 n_codebooks, u32 audio_vocab, u32 audio_pad_id, u32 n_seq,
  per sequence (u32 n, i32 spk_pos or -1, u32 spk_dim or 0), per sequence its ids [n][W] as f32
  then its speaker [spk_dim] f32, then per event (sequence, t, codebook order) audio_vocab f32
  log-probabilities.
"""
from __future__ import annotations

import math
import struct
from dataclasses import dataclass

import numpy as np

MAGIC, VERSION = b"Z2KLDIV2", 2


@dataclass
class Sequence:
    ids: np.ndarray                     # [n][n_codebooks + 1] input rows
    spk: np.ndarray | None = None       # [spk_dim] speaker embedding, or None
    spk_pos: int = -1


def log_softmax(logits: np.ndarray) -> np.ndarray:
    """Rows of f32 log-probabilities the way the reference computes them: the max in f32, the
    sum of exp(logit - max) in f64, lse = max + f32(log(sum)), logp = logit - lse in f32."""
    x = np.asarray(logits, np.float32)
    mx = x.max(-1, keepdims=True)
    se = np.exp((x - mx).astype(np.float64)).sum(-1, keepdims=True)
    lse = mx + np.log(se).astype(np.float32)
    return (x - lse).astype(np.float32)


def events(seq_ids: np.ndarray, logits: np.ndarray, n_codebooks: int, audio_vocab: int, pad: int):
    """(log-probabilities [E][audio_vocab], labels [E], codebook [E], skipped) of one sequence, in
    (t, codebook) order. logits: [n][n_codebooks][audio_vocab]."""
    ids = np.asarray(seq_ids)
    n = ids.shape[0]
    lab = np.rint(np.asarray(ids[1:, :n_codebooks], np.float64)).astype(np.int64)   # [n-1][ncb]
    keep = (lab != pad) & (lab >= 0) & (lab < audio_vocab)
    t_idx, cb_idx = np.nonzero(keep)                 # row-major: t, then codebook
    lp = log_softmax(np.asarray(logits)[: n - 1][t_idx, cb_idx])
    return lp, lab[t_idx, cb_idx], cb_idx, int((~keep).sum())


def _logits(model, s: Sequence):
    ids = np.rint(np.asarray(s.ids, np.float64)).astype(np.int32)     # base files carry f32 ids
    spk_pos = s.spk_pos if s.spk_pos >= 0 else 0
    return model.logits(ids, s.spk, spk_pos) if s.spk is not None else model.logits(ids)


def perplexity(model, seqs: list[Sequence]) -> dict:
    """Teacher-forced perplexity of `model` (runtime.Model) over the sequences."""
    hp = model.hp
    ncb, av, pad = hp.n_codebooks, hp.audio_vocab, hp.audio_pad_id
    nll, cnt, skipped = np.zeros(ncb), np.zeros(ncb, np.int64), 0
    for s in seqs:
        lp, lab, cb, sk = events(s.ids, _logits(model, s), ncb, av, pad)
        skipped += sk
        np.add.at(nll, cb, -lp[np.arange(len(lab)), lab].astype(np.float64))
        np.add.at(cnt, cb, 1)
    tot = int(cnt.sum())
    if tot == 0:
        raise ValueError("no events scored")
    mean = float(nll.sum() / tot)
    return {"events": tot, "skipped": skipped, "ppl": math.exp(mean), "mean_nll": mean,
            "ppl_per_codebook": [math.exp(nll[c] / cnt[c]) if cnt[c] else 0.0 for c in range(ncb)],
            "events_per_codebook": cnt.tolist()}


def kl_base(model, seqs: list[Sequence], path: str) -> dict:
    """Write the reference model's event log-probabilities to `path`; returns its perplexity."""
    hp = model.hp
    ncb, av, pad = hp.n_codebooks, hp.audio_vocab, hp.audio_pad_id
    nll, n_ev, skipped = 0.0, 0, 0
    with open(path, "wb") as f:
        f.write(MAGIC + struct.pack("<5I", VERSION, ncb, av, pad, len(seqs)))
        for s in seqs:
            f.write(struct.pack("<IiI", len(s.ids), s.spk_pos if s.spk is not None else -1,
                                0 if s.spk is None else len(s.spk)))
        for s in seqs:
            f.write(np.asarray(s.ids, np.float32).tobytes())
            if s.spk is not None:
                f.write(np.asarray(s.spk, np.float32).tobytes())
        for s in seqs:
            lp, lab, _, sk = events(s.ids, _logits(model, s), ncb, av, pad)
            f.write(lp.astype(np.float32).tobytes())
            nll += float(-lp[np.arange(len(lab)), lab].astype(np.float64).sum())
            n_ev += len(lab)
            skipped += sk
    if n_ev == 0:
        raise ValueError("no events scored")
    return {"events": n_ev, "skipped": skipped, "ppl_ref": math.exp(nll / n_ev)}


def read_base(path: str) -> tuple[dict, list[Sequence], np.ndarray]:
    """Header, sequences and the [E][audio_vocab] event log-probabilities of a base file (the
    event block memory-mapped: bases of large corpora run to gigabytes)."""
    with open(path, "rb") as f:
        head = f.read(28)
        if len(head) < 28 or head[:8] != MAGIC:
            raise ValueError(f"{path}: bad magic")
        version, ncb, av, pad, n_seq = struct.unpack_from("<5I", head, 8)
        if version != VERSION:
            raise ValueError(f"{path}: version {version} != {VERSION} (regenerate base)")
        meta = [struct.unpack("<IiI", f.read(12)) for _ in range(n_seq)]
        seqs = []
        for n, spk_pos, sdim in meta:
            ids = np.frombuffer(f.read(4 * n * (ncb + 1)), np.float32).reshape(n, ncb + 1).copy()
            spk = np.frombuffer(f.read(4 * sdim), np.float32).copy() if sdim else None
            seqs.append(Sequence(ids, spk, spk_pos))
        off = f.tell()
        size = f.seek(0, 2)
    if (size - off) % (4 * av):
        raise ValueError(f"{path}: truncated event block")
    n_ev = (size - off) // (4 * av)
    lp = np.memmap(path, np.float32, "r", off, (n_ev, av)) if n_ev else np.zeros((0, av), np.float32)
    return {"n_codebooks": ncb, "audio_vocab": av, "audio_pad_id": pad}, seqs, lp


def kl_divergence(model, path: str) -> dict:
    """Score `model` against a base file: KLD(ref || test) per event with its quantiles, top-1
    agreement, the true label's log-probability difference and both perplexities."""
    hp = model.hp
    head, seqs, ref_all = read_base(path)
    ncb, av, pad = hp.n_codebooks, hp.audio_vocab, head["audio_pad_id"]
    if head["n_codebooks"] != ncb or head["audio_vocab"] != av:
        raise ValueError(f"base/model mismatch: base ncb={head['n_codebooks']} av={head['audio_vocab']}, "
                         f"model ncb={ncb} av={av}")
    kld_all, cb_all, agree_all, ref_nll, test_nll, dlp = [], [], [], 0.0, 0.0, []
    e0 = 0
    for s in seqs:
        lp, lab, cb, _ = events(s.ids, _logits(model, s), ncb, av, pad)
        ref = ref_all[e0:e0 + len(lab)]
        if len(ref) != len(lab):
            raise ValueError(f"{path}: truncated event block")
        e0 += len(lab)
        kld = (np.exp(ref.astype(np.float64)) * (ref.astype(np.float64) - lp)).sum(-1)
        kld_all.append(np.maximum(kld, 0.0))
        cb_all.append(cb)
        agree_all.append(ref.argmax(-1) == lp.argmax(-1))
        r = np.arange(len(lab))
        ref_nll += float(-ref[r, lab].astype(np.float64).sum())
        test_nll += float(-lp[r, lab].astype(np.float64).sum())
        dlp.append(lp[r, lab].astype(np.float64) - ref[r, lab].astype(np.float64))
    kld, cb, agree, dlp = (np.concatenate(x) for x in (kld_all, cb_all, agree_all, dlp))
    n = len(kld)
    if n == 0:
        raise ValueError("no events scored")
    srt = np.sort(kld)

    def q(p):
        return float(srt[int(round(p * (n - 1)))])

    ppl_ref, ppl_test = math.exp(ref_nll / n), math.exp(test_nll / n)
    return {"events": n, "ppl_ref": ppl_ref, "ppl_test": ppl_test, "ppl_ratio": ppl_test / ppl_ref,
            "kld_mean": float(kld.mean()), "kld_median": q(0.5), "kld_p90": q(0.9), "kld_p95": q(0.95),
            "kld_p99": q(0.99), "kld_max": float(srt[-1]), "kld_min": float(srt[0]),
            "top1_agreement": float(agree.mean()), "dlogp_mean": float(dlp.mean()),
            "dlogp_rms": float(np.sqrt((dlp ** 2).mean())),
            "kld_mean_per_codebook": [float(kld[cb == c].mean()) if (cb == c).any() else 0.0 for c in range(ncb)],
            "top1_per_codebook": [float(agree[cb == c].mean()) if (cb == c).any() else 0.0 for c in range(ncb)]}
