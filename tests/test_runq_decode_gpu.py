"""The device-resident decode of runq models (mvb_runq_load + the mvb_qwen_* step calls) against runq.c itself.

runq.c's forward (runq.c:477-614) is restated kernel by kernel: the int8 / fp32-scale matvecs are bit-exact given
their activations, and every other operation keeps runq.c's order and rounding (its quantize by division, rmsnorm
with eps 1e-5, interleaved RoPE from the host C library's powf/cosf/sinf, softmax and SiLU with the host's expf).
The bar is therefore bit-identical logits at every position and identical greedy token ids for the whole run.

The references are the committed fixture made by runq.c (tests/golden/runq_tiny.npz) and runq.c's CPU build in
oracle/_ref (built where the reference tree is available; it travels with the working tree)."""
import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT, golden, load_pkg

pytestmark = pytest.mark.gpu
REF = os.path.join(ROOT, "oracle", "_ref")


def need_ref():
    if not os.path.exists(os.path.join(REF, "libref_runq.so")):
        pytest.fail("oracle/_ref/libref_runq.so is missing: run make -C oracle ref where the reference exists")


def ref_greedy(model, prompt, npos, tmp_path):
    """runq.c's CPU build (its own forward and sample_argmax) on `model`: (ids after the prompt, logits per
    position), in a child process because the harness keeps one model per process."""
    need_ref()
    out = str(tmp_path / "ref_logits.npy")
    code = (f"import sys, numpy as np\nsys.path.insert(0, {os.path.join(ROOT, 'oracle')!r})\nimport oracle\n"
            f"r = oracle.RefRunq()\nr.open({model!r})\nids, lg = r.greedy({list(prompt)!r}, {npos})\n"
            f"np.save({out!r}, lg)\nprint(','.join(map(str, ids)))\n")
    r = subprocess.run(["python", "-c", code], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr
    return [int(t) for t in r.stdout.strip().split(",") if t], np.load(out)


def device_logits(dec, prompt, ids, npos):
    """Logits of positions 0 .. npos-1, feeding the prompt and then `ids` (the reference's greedy ids)."""
    seq = list(prompt) + list(ids)
    return np.stack([dec.forward(seq[p], p)[1] for p in range(npos)])


def assert_bits(ours, ref):
    same = ours.view(np.uint32) == ref.view(np.uint32)
    if not same.all():
        pos, row = np.argwhere(~same)[0]
        pytest.fail(f"{int((~same).sum())} logits differ; first at position {pos}, row {row}: "
                    f"{ours[pos, row]!r} vs {ref[pos, row]!r}")


def test_runq_tiny_vs_golden(tmp_path):
    """Head size 32, two layers: the fixture that runq.c itself wrote."""
    mvb = load_pkg()
    z = golden("runq_tiny.npz")
    path = str(tmp_path / "tiny.bin")
    mvb.qwb.write_synthetic_runq(path, mvb.qwb.RUNQ_TINY, seed=int(z["seed"]), gs=int(z["gs"]))
    dec = mvb.RunqDecoder(path, ctx=64)
    try:
        prompt, ids = [int(t) for t in z["prompt"]], [int(t) for t in z["ids"]]
        assert dec.cfg["head_k"] == dec.cfg["vocab_size"] == 300
        assert_bits(device_logits(dec, prompt, ids, z["logits"].shape[0]), z["logits"])
        got = dec.generate(prompt, len(ids))
        stop = ids.index(1) if 1 in ids else len(ids)  # runq.c stops before BOS
        assert got.tolist() == ids[:stop]
    finally:
        dec.close()


@pytest.mark.parametrize("cfg_name, gs, npos", [("STORIES15M", 32, 256), ("STORIES110M", 32, 300),
                                                ("STORIES110M", 64, 160)])
def test_runq_stories_vs_reference(tmp_path, cfg_name, gs, npos):
    """Configs 1 and 2 (stories15M / stories110M architectures, shared classifier, 4 seeded prompt ids) at group
    size 32, and stories110M at the group size the reference's own converter gives it (tools/bin2q80.py:44-46
    takes 64 when it divides dim): the logits of every position bit for bit (past 256 positions the attention
    stages its cached values in a second chunk), then the greedy ids of the whole run."""
    mvb = load_pkg()
    cfg = getattr(mvb.qwb, cfg_name)
    path = str(tmp_path / f"{cfg_name}_g{gs}.bin")
    mvb.qwb.write_synthetic_runq(path, cfg, seed=3, gs=gs)
    prompt = [int(t) for t in np.random.default_rng(4).integers(3, cfg["vocab_size"], 4)]
    ref_ids, ref_logits = ref_greedy(path, prompt, npos, tmp_path)
    dec = mvb.RunqDecoder(path, ctx=cfg["seq_len"])
    try:
        assert_bits(device_logits(dec, prompt, ref_ids, npos), ref_logits)
        got = dec.generate(prompt, npos - len(prompt) + 1)
        stop = ref_ids.index(1) if 1 in ref_ids else len(ref_ids)
        assert got.tolist() == ref_ids[:stop]
    finally:
        dec.close()


@pytest.mark.parametrize("gs", [32, 64])
def test_runq_grouped_query_and_separate_classifier(tmp_path, gs):
    """Fewer kv heads than query heads (kv_mul 2, runq.c:483-484), head size 48, and a classifier stored apart from
    the embedding (shared_classifier 0, runq.c:315), at both group sizes."""
    mvb = load_pkg()
    cfg = dict(dim=192, hidden_dim=512, n_layers=3, n_heads=4, n_kv_heads=2, vocab_size=1000, seq_len=128)
    path = str(tmp_path / "gqa.bin")
    mvb.qwb.write_synthetic_runq(path, cfg, seed=8, gs=gs, shared=False)
    prompt = [5, 77, 901, 12, 400]
    ref_ids, ref_logits = ref_greedy(path, prompt, 40, tmp_path)
    dec = mvb.RunqDecoder(path, ctx=128)
    try:
        assert_bits(device_logits(dec, prompt, ref_ids, 40), ref_logits)
    finally:
        dec.close()


def test_runq_odd_group_counts(tmp_path):
    """Odd group counts per row (dim 544: 17 groups; hidden 1120: 35), whose per-CTA scale arrays need padding to
    keep the product rows 16-byte aligned for the fold's 16-byte loads; head size 32."""
    mvb = load_pkg()
    cfg = dict(dim=544, hidden_dim=1120, n_layers=2, n_heads=17, n_kv_heads=17, vocab_size=700, seq_len=64)
    path = str(tmp_path / "odd.bin")
    mvb.qwb.write_synthetic_runq(path, cfg, seed=12, gs=32)
    prompt = [9, 300, 41]
    ref_ids, ref_logits = ref_greedy(path, prompt, 24, tmp_path)
    dec = mvb.RunqDecoder(path, ctx=64)
    try:
        assert_bits(device_logits(dec, prompt, ref_ids, 24), ref_logits)
    finally:
        dec.close()


def test_runq_bytes_and_file_loaders_agree(tmp_path):
    """mvb_runq_load (caller's bytes) and mvb_runq_load_file (mapped file) give the same model."""
    mvb = load_pkg()
    path = str(tmp_path / "tiny.bin")
    mvb.qwb.write_synthetic_runq(path, mvb.qwb.RUNQ_TINY, seed=21, gs=32)
    a = mvb.RunqDecoder(path, ctx=32)
    b = mvb.RunqDecoder(open(path, "rb").read(), ctx=32)
    try:
        for pos, tok in enumerate([3, 9, 200, 17]):
            ra, la = a.forward(tok, pos)
            rb, lb = b.forward(tok, pos)
            assert ra == rb and np.array_equal(la.view(np.uint32), lb.view(np.uint32))
            assert ra == int(np.argmax(la))
    finally:
        a.close()
        b.close()


def test_runq_load_rejections(tmp_path):
    mvb = load_pkg()
    path = str(tmp_path / "tiny.bin")
    size = mvb.qwb.write_synthetic_runq(path, mvb.qwb.RUNQ_TINY, seed=1, gs=32)
    data = open(path, "rb").read()
    with pytest.raises(mvb.MatvecError, match="header describes"):
        mvb.RunqDecoder(data[:size - 1], ctx=32)
    with pytest.raises(mvb.MatvecError, match="not a runq version 2"):
        mvb.RunqDecoder(b"XXXX" + data[4:], ctx=32)
    with pytest.raises(mvb.MatvecError, match="not a runq version 2"):
        mvb.RunqDecoder(data[:100], ctx=32)
    g16 = str(tmp_path / "g16.bin")
    mvb.qwb.write_synthetic_runq(g16, mvb.qwb.RUNQ_TINY, seed=1, gs=16)  # runq.c's FPGA build refuses it too
    with pytest.raises(mvb.MatvecError, match="group size 32 or 64"):
        mvb.RunqDecoder(g16, ctx=32)
    with pytest.raises(mvb.MatvecError, match="cannot map"):
        mvb.RunqDecoder(str(tmp_path / "missing.bin"), ctx=32)
    # a .qwb is not a runq checkpoint, and the other way round
    with pytest.raises(mvb.MatvecError, match="not a .qwb"):
        mvb.QwenDecoder(path, ctx=32)
