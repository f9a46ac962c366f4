"""Host-side logic of the drop-in boundary, without a GPU: validation, packing, sharding."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from onyx_b200 import bitmask, masked_selection, torch_backend, torch_grammar_mask, vocab_parallel
from onyx_b200 import workloads


def test_pack_ids_matches_pack_bool_and_unpack():
    rng = np.random.default_rng(0)
    for v in (1, 31, 32, 33, 100, 151665):
        valid = rng.random(v) < 0.1
        valid[rng.integers(0, v)] = True
        ids = np.flatnonzero(valid)
        a = bitmask.pack_ids(ids, v)
        b = bitmask.pack_bool(valid)
        assert a.shape == (bitmask.words_for(v),)
        assert np.array_equal(a, b)
        assert np.array_equal(bitmask.unpack(a, v), valid)
        # tail bits stay zero
        if v % 32:
            assert int(a[-1]) >> (v % 32) == 0


def test_pack_ids_rejects_out_of_range():
    with pytest.raises(ValueError):
        bitmask.pack_ids([5], 5)
    with pytest.raises(ValueError):
        bitmask.pack_ids([-1], 5)


def test_valid_id_validation_mirrors_reference():
    v = torch_grammar_mask._validate_valid_token_ids
    err = torch_grammar_mask.TorchGrammarMaskInvariantError
    for bad, msg in (
        ([1, 2], "must be a tuple"),
        ((), "cannot be empty"),
        ((1, True), "only Python integers"),
        ((1, 9), "outside vocabulary range"),
        ((2, 1), "strictly increasing"),
        ((1, 1), "strictly increasing"),
    ):
        with pytest.raises(err, match=msg):
            v(bad, 5)
    v((0, 4), 5)


def test_factory_validation_and_unavailable_device():
    create = torch_grammar_mask.create_cuda_grammar_logit_mask
    with pytest.raises(TypeError):
        create(True)
    with pytest.raises(ValueError):
        create(0)
    with pytest.raises(ValueError):
        create(4, device_index=-1)
    with pytest.raises(TypeError):
        create(4, clock=3)
    if not torch.cuda.is_available():
        with pytest.raises(torch_grammar_mask.TorchGrammarMaskUnavailableError):
            create(4)


def test_selector_rejects_bad_rows_before_touching_a_device():
    sel = torch_backend.select_cuda_argmax
    with pytest.raises(torch_backend.TorchBackendInvariantError, match="nonempty"):
        sel(torch.zeros(0))
    with pytest.raises(torch_backend.TorchBackendInvariantError, match="nonempty"):
        sel(torch.zeros(2, 3))
    with pytest.raises(torch_backend.TorchBackendInvariantError, match="non-CUDA"):
        sel(torch.zeros(3))


def test_batched_entry_points_reject_cpu_tensors():
    with pytest.raises(ValueError, match="CUDA"):
        masked_selection.masked_argmax(torch.zeros(2, 8))
    with pytest.raises(TypeError):
        masked_selection.dtype_code(torch.int32)
    assert masked_selection.mask_words(32) == 1 and masked_selection.mask_words(33) == 2


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_bounds_cover_everything_and_align(world):
    for rows in (0, 1, 7, 64, 1024):
        spans = [vocab_parallel.batch_shard_bounds(rows, r, world) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == rows
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    for vocab in (1, 31, 32000, 128256, 151665, 256000):
        spans = [vocab_parallel.vocab_shard_bounds(vocab, r, world) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == vocab
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        # every non-empty shard starts on a mask-word boundary
        assert all(lo % 32 == 0 for lo, hi in spans if hi > lo)


def _oracle_keys(logits_bits, masks, lo, hi):
    """Pack oracle shard partials into the library's 64-bit key format (test helper)."""
    part = oracle.vocab_shard_select(logits_bits[:, lo:hi], masks[:, lo // 32 : (hi + 31) // 32], lo,
                                     dtype="bf16")
    keys = []
    for p in part:
        if not p.found and not p.nan:
            keys.append(0)
        elif p.nan:
            keys.append((0xFFFFFFFF << 32) | 0)
        else:
            f = np.float32(p.best)
            u = int(np.array([0.0 if f == 0 else f], np.float32).view(np.uint32)[0])
            order = (~u & 0xFFFFFFFF) if u >> 31 else (u | 0x80000000)
            keys.append((order << 32) | (0xFFFFFFFF - int(p.idx)))
    return keys


@pytest.mark.parametrize("world", [2, 3, 8])
def test_host_combine_of_shard_keys_equals_unsharded_oracle(world):
    rng = np.random.default_rng(7)
    rows, vocab = 9, 1000
    x = workloads.normal_bf16(rng, (rows, vocab))
    # ties across shard boundaries and an all -inf row
    x[0, 10] = x[0, 600] = workloads.bf16_bits(np.array([100.0], np.float32))[0]
    x[3, :] = 0xFF80
    masks = workloads.bernoulli_masks(rng, np.full(rows, 0.2), vocab)
    masks[0, 10 // 32] |= np.uint32(1 << (10 % 32))
    masks[0, 600 // 32] |= np.uint32(1 << (600 % 32))
    masks[5, :] = 0
    keys = [
        _oracle_keys(x, masks, *vocab_parallel.vocab_shard_bounds(vocab, r, world))
        for r in range(world)
    ]
    got = vocab_parallel.combine_keys_host(keys)
    idx, st = oracle.masked_argmax(x, masks, dtype="bf16")
    for r in range(rows):
        assert got[r][1] == int(st[r])
        if int(st[r]) in (0, 2):
            assert got[r][0] == int(idx[r])
    assert got[0][0] == 10 and got[5][1] == masked_selection.STATUS_EMPTY_MASK


def test_workload_shapes_and_determinism():
    a = workloads.batched(rows=4, vocab=1000)
    b = workloads.batched(rows=4, vocab=1000)
    assert np.array_equal(a["logits_bf16"], b["logits_bf16"])
    assert np.array_equal(a["masks"], b["masks"])
    assert a["masks"].shape == (4, 32)
    dens = bitmask.unpack(a["masks"], 1000).mean(axis=1)
    assert np.all(dens > 0)
    v = workloads.synthetic_vocabulary(np.random.default_rng(1), 1000)
    assert len(v) == 1000 and all(len(t) == 1 for t in v[:256])
    assert all(2 <= len(t) <= 8 and all(0x20 <= c < 0x7F for c in t) for t in v[256:])


def _prmt_sign(word: int, sel: int) -> int:
    """prmt.b32 d, word, 0, sel with every selector nibble in sign-replicate mode: byte n of
    d is 0xFF when bit 7 of byte (nibble n & 3) of `word` is set, else 0x00."""
    out = 0
    for n in range(4):
        src = (sel >> (4 * n)) & 0x3
        if (word >> (8 * src + 7)) & 1:
            out |= 0xFF << (8 * n)
    return out


def test_mask_expansion_multiplies_are_carry_free():
    """The device expansion of 8 mask bits into four packed 16-bit lane masks
    (expand8_16 in onyx_common.cuh) for every byte value, with the unmasked high bits a
    shifted mask word leaves above the byte."""
    for byte in range(256):
        for above in (0, 0xABCDEF00, 0xFFFFFF00):
            bits = byte | above
            lo = ((bits & 0x0F) * 0x10204080) & 0xFFFFFFFF
            hi = ((bits & 0xF0) * 0x01020408) & 0xFFFFFFFF
            got = [_prmt_sign(lo, 0x9988), _prmt_sign(lo, 0xBBAA),
                   _prmt_sign(hi, 0x9988), _prmt_sign(hi, 0xBBAA)]
            want = []
            for pair in range(4):
                b0 = (byte >> (2 * pair)) & 1
                b1 = (byte >> (2 * pair + 1)) & 1
                want.append((0xFFFF if b0 else 0) | (0xFFFF0000 if b1 else 0))
            assert got == want, (byte, above)


def test_dfa_mask_host_helpers():
    from onyx_b200 import dfa_masks
    data, offsets = dfa_masks.pack_tokens([b"ab", b"", b"c"])
    assert data.tolist() == [0x61, 0x62, 0x63] and offsets.tolist() == [0, 2, 2, 3]
    trans = np.zeros((3, 256), np.int32)
    assert dfa_masks.dead_is_absorbing(trans, 0)
    trans[0, 7] = 2
    assert not dfa_masks.dead_is_absorbing(trans, 0)
    # shape and argument errors are raised on the host, before any device is touched
    with pytest.raises(ValueError):
        dfa_masks.DfaMaskBuilder(np.zeros((3, 255), np.int32), 0, [b"a"])
    with pytest.raises(ValueError):
        dfa_masks.DfaMaskBuilder(trans, 3, [b"a"])
    with pytest.raises(ValueError):
        dfa_masks.DfaMaskBuilder(trans, 0, [])
    with pytest.raises(ValueError):
        dfa_masks.DfaMaskBuilder(trans, 0, [b"a"], device="cpu")


def test_digits_dfa_matches_the_restated_regex_compiler():
    """The config-1 grammar's table, built directly in workloads, gives the same valid-token
    sets as the oracle's compile of [0-9]{1,8} (state numbering aside): from the start
    state over the synthetic 32,000-token vocabulary and over hand-picked tokens, and after
    every prefix of digits."""
    from types import SimpleNamespace

    from oracle.regex_dfa import compile_regex_dfa

    ref = compile_regex_dfa("[0-9]{1,8}")
    d = workloads.digits_dfa(8)
    mine = SimpleNamespace(trans=d["trans"], dead=d["dead"])
    vocab = workloads.single_row()["vocabulary"] + [
        b"5", b"5a", b"5ab", b"12345678", b"123456789", b"1234567890", b"a", b"0x", b"00", b"9 ",
    ]
    assert np.array_equal(oracle.dfa_scan_bitmask(mine, d["start"], vocab),
                          oracle.dfa_scan_bitmask(ref, ref.start, vocab))
    for k in range(1, 9):
        s_ref = ref.walk(ref.start, b"7" * k)
        s_mine = d["start"]
        for b in b"7" * k:
            s_mine = int(d["trans"][s_mine, b])
        assert np.array_equal(oracle.dfa_scan_bitmask(mine, s_mine, vocab),
                              oracle.dfa_scan_bitmask(ref, s_ref, vocab))


def test_bench_shards_and_records_are_consistent():
    """The bench's config 5a splits 1,024 rows over the ranks, its traffic figures scale with
    the shard, and both arms print the same config object."""
    import bench

    for world in (1, 2, 4, 8):
        assert bench.rows_per_gpu("scaling", world) * world == 1024
        assert bench.rows_per_gpu("batched", world) == 64
        t = bench.traffic_per_launch("vocab_parallel", world)
        assert t == pytest.approx(bench.NCU_TRAFFIC_PER_LAUNCH["vocab_parallel"] / world)
        # captured traffic stays within 2 % above the algorithmic bytes of the same launch
        for name in ("batched", "table_gather", "spec_verify", "scaling", "vocab_parallel"):
            rows = bench.rows_per_gpu(name, world) if name != "vocab_parallel" else 1024
            algo = bench.bytes_per_row(name, world) * rows
            ratio = bench.traffic_per_launch(name, world) / algo
            assert 1.0 <= ratio < 1.02, (name, world, ratio)
        cfg = bench.workload_config("scaling", world, "peer")
        assert cfg["rows_per_step_per_gpu"] == 1024 // world
        assert cfg == bench.workload_config("scaling", world, "peer")
    assert bench.traffic_per_launch("no such workload", 1) is None


def test_reference_arm_prints_the_contract_line():
    """`bench.py --impl reference` times the CPU restatement and prints one JSON line with the
    GPU arm's metric, unit and config."""
    import json
    import subprocess
    import sys
    from pathlib import Path

    import bench

    root = Path(__file__).resolve().parents[1]
    out = subprocess.run([sys.executable, str(root / "bench.py"), "--impl", "reference",
                          "--steps", "2", "--warmup", "3"], cwd=root, capture_output=True,
                         text=True, timeout=300, check=True).stdout
    lines = [json.loads(x) for x in out.splitlines() if x.startswith("{")]
    assert len(lines) == 1
    line = lines[0]
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC
    assert line["unit"] == bench.UNIT and line["higher_is_better"] is True
    assert line["config"] == bench.workload_config("batched", 1, "peer")
    assert line["value"] > 0 and line["cpu_baseline"]["kind"] == "port"
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
