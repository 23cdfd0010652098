"""Checkpoint format and token loader (CPU only).

The checkpoint bytes are checked against the layout the reference documents
for BinaryCheckpoint (Sources/Core/Module.swift:4838-4852), field by field,
and the loader's rejections against its reader (Module.swift:4908-4992): bad
magic, unsupported version, truncation anywhere, implausible rank, trailing
bytes; version-1 files (no buffer section) load. The token loader follows
MemoryMappedTokenDataset (Sources/Core/Data.swift:1827-2000).
"""
import struct

import numpy as np
import pytest

from magma_b200 import checkpoint as ck
from magma_b200.data import MemoryMappedTokenDataset, TokenDatasetError, write_token_file


def test_checkpoint_bytes_follow_the_documented_layout():
    got = ck.encode([ck.Entry("w", (2,), [1.0, -2.0])], [ck.Entry("s", (), [3.0])])
    want = (b"STCHKPT\x00" + struct.pack("<I", 2)
            + struct.pack("<I", 1) + struct.pack("<I", 1) + b"w" + struct.pack("<II", 1, 2)
            + struct.pack("<ff", 1.0, -2.0)
            + struct.pack("<I", 1) + struct.pack("<I", 1) + b"s" + struct.pack("<I", 0)
            + struct.pack("<f", 3.0))
    assert got == want


def test_checkpoint_round_trip(tmp_path):
    rng = np.random.default_rng(0)
    params = [ck.Entry("h0.qkv_w", (6, 4), rng.standard_normal(24)),
              ck.Entry("bias", (4,), rng.standard_normal(4)),
              ck.Entry("gewicht-ü", (2, 1, 3), rng.standard_normal(6)),
              ck.Entry("scalar", (), [2.5])]
    bufs = [ck.Entry("running", (3,), [1, 2, 3])]
    ck.save(tmp_path / "c.bin", params, bufs)
    version, p2, b2 = ck.load(tmp_path / "c.bin")
    assert version == 2 and len(p2) == 4 and len(b2) == 1
    for a, b in zip(params + bufs, p2 + b2):
        assert a.name == b.name and a.shape == b.shape
        assert np.array_equal(a.values, b.values)


def test_version1_files_load_without_buffers():
    data = ck.encode([ck.Entry("w", (3,), [1, 2, 3])], version=1)
    version, params, bufs = ck.decode(data)
    assert version == 1 and bufs == [] and params[0].values.tolist() == [1, 2, 3]


def test_corrupt_files_are_rejected():
    good = ck.encode([ck.Entry("w", (2, 2), [1, 2, 3, 4])], [ck.Entry("b", (1,), [5])])
    ck.decode(good)
    for cut in range(len(good)):  # truncated anywhere
        with pytest.raises(ck.CheckpointError):
            ck.decode(good[:cut])
    with pytest.raises(ck.CheckpointError, match="trailing"):
        ck.decode(good + b"\x00")
    with pytest.raises(ck.CheckpointError, match="magic"):
        ck.decode(b"NOTCKPT\x00" + good[8:])
    with pytest.raises(ck.CheckpointError, match="version"):
        ck.decode(good[:8] + struct.pack("<I", 3) + good[12:])
    bad_rank = (b"STCHKPT\x00" + struct.pack("<II", 2, 1) + struct.pack("<I", 1) + b"w"
                + struct.pack("<I", 65))
    with pytest.raises(ck.CheckpointError, match="rank"):
        ck.decode(bad_rank)


def test_shape_mismatch_is_reported():
    e = [ck.Entry("w", (2, 3), np.zeros(6))]
    ck.match(e, [("w", (2, 3))], "parameter")
    with pytest.raises(ck.CheckpointError, match="shape"):
        ck.match(e, [("w", (3, 2))], "parameter")
    with pytest.raises(ck.CheckpointError, match="count"):
        ck.match(e, [("w", (2, 3)), ("b", (3,))], "parameter")


def test_token_dataset_samples_and_batches(tmp_path):
    toks = (np.arange(1000) * 53) % 50257  # ids above 255 exercise both bytes
    write_token_file(tmp_path / "t.bin", toks)
    ds = MemoryMappedTokenDataset(tmp_path / "t.bin", 8)
    assert ds.token_count == 1000 and len(ds) == 992
    x, y = ds.get_sample(5)
    assert x.dtype == np.int32 and x.tolist() == toks[5:13].tolist()
    assert y.tolist() == toks[6:14].tolist()
    seq = list(ds.batches(100, shuffle=False))
    assert len(seq) == 9  # 992 samples: the partial tenth batch is dropped
    assert np.array_equal(seq[1][0][3], toks[103:111])
    a = [b[0].copy() for b in ds.batches(64, shuffle=True, seed=7)]
    b = [b[0].copy() for b in ds.batches(64, shuffle=True, seed=7)]
    assert all(np.array_equal(u, w) for u, w in zip(a, b))
    firsts = np.concatenate([u[:, 0] for u in a])
    assert len(set(firsts.tolist())) == len(firsts)  # a permutation: no sample twice
    with pytest.raises(IndexError):
        ds.get_sample(992)


def test_token_dataset_rejects_small_or_missing_files(tmp_path):
    write_token_file(tmp_path / "small.bin", np.arange(8))
    with pytest.raises(TokenDatasetError, match="too small"):
        MemoryMappedTokenDataset(tmp_path / "small.bin", 8)
    with pytest.raises(TokenDatasetError, match="not found"):
        MemoryMappedTokenDataset(tmp_path / "missing.bin", 8)


def test_gpt_checkpoint_order_is_the_reference_parameter_list():
    """GPT2.parameters() (Benchmarks/GPT2Shakespeare/Sources/main.swift:255-256,
    184-185, 127-130, 314-317): wte, wpe, 16 tensors per block (ln1, wQ, wK, wV,
    wO, ln2, cFc, cProj; weight then bias), lnF, lmHead (no bias)."""
    from magma_b200.gpt import gpt2_small

    cfg = gpt2_small()
    ref = cfg.reference_parameters()
    D, V = 768, 50257
    per_block = [(D,), (D,), (D, D), (D,), (D, D), (D,), (D, D), (D,), (D, D), (D,), (D,), (D,),
                 (4 * D, D), (4 * D,), (D, 4 * D), (D,)]
    want = [(V, D), (1024, D)] + per_block * 12 + [(D,), (D,), (V, D)]
    assert len(ref) == 2 + 16 * 12 + 3 == 197
    assert [s for _, s, _ in ref] == want
    assert [n for n, _, _ in ref][:6] == ["weight", "weight", "weight", "bias", "weight", "bias"]
    # parameters of the reference model: 163M with its separate lm-head
    assert sum(int(np.prod(s)) for _, s, _ in ref) == 124_439_808 + V * D


@pytest.mark.parametrize("tied", [True, False])
def test_gpt_checkpoint_entries_round_trip(tmp_path, tied):
    from magma_b200.gpt import GPTConfig

    cfg = GPTConfig(vocab=70, seq=16, layers=2, heads=2, dim=32, tied=tied)
    total = cfg.offsets()["__total__"][0]
    rng = np.random.default_rng(1)
    arena = np.zeros(total, np.float32)  # alignment gaps and vocabulary padding stay zero
    for _, shp, off in cfg.reference_parameters():
        n = int(np.prod(shp))
        arena[off:off + n] = rng.standard_normal(n)
    ents = cfg.to_reference_entries(arena)
    ck.save(tmp_path / "g.bin", ents)
    _, back, _ = ck.load(tmp_path / "g.bin")
    # wQ of layer 0 is the first D rows of the fused projection
    q_off = cfg.offsets()["h0.qkv_w"][0]
    assert np.array_equal(back[4].values, arena[q_off:q_off + 32 * 32])
    k_off = q_off + 32 * 32
    assert np.array_equal(back[6].values, arena[k_off:k_off + 32 * 32])
    got = np.zeros_like(arena)
    cfg.from_reference_entries(back, got)
    assert np.array_equal(got, arena)
    with pytest.raises(ck.CheckpointError, match="count"):
        cfg.from_reference_entries(back[:-1], got)
    if tied:
        bad = list(back)
        bad[-1] = ck.Entry("weight", bad[-1].shape, bad[-1].values + 1)
        with pytest.raises(ck.CheckpointError, match="untied"):
            cfg.from_reference_entries(bad, got)
