"""The device-resident decode (mvb_qwen_*) against qwen.c itself.

Every matvec in the decode is bit-exact given its activations, and the rest of the step follows qwen.c's
operation order and rounding, expf included (the device reproduces the host C library's expf on every float).
The bar: greedy token ids identical to qwen.c for the whole run, and logits bit-identical to qwen.c's at every
position (the largest difference is printed when they are not)."""
import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT, golden, load_pkg

pytestmark = pytest.mark.gpu
REF = os.path.join(ROOT, "oracle", "_ref")


def ref_run(model, prompt, n, ctx, dump):
    r = subprocess.run([os.path.join(REF, "qwen"), model, "--ids", ",".join(map(str, prompt)), "-t", "0", "-n", str(n),
                        "-c", str(ctx), "--logits", dump], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr
    return [int(t) for t in r.stdout.strip().split(",") if t]


def compare_logits(ours, ref):
    diff = np.abs(ours.astype(np.float64) - ref.astype(np.float64))
    exact = float(np.mean(ours.view(np.uint32) == ref.view(np.uint32)))
    print(f"max |diff| {diff.max():.3e}, max rel {np.max(diff / np.maximum(np.abs(ref), 1e-30)):.3e}, "
          f"bit-identical fraction {exact:.6f}")
    assert np.array_equal(ours.view(np.uint32), ref.view(np.uint32))


def test_tiny_decode_vs_golden(tmp_path):
    mvb = load_pkg()
    z = golden("qwen_tiny.npz")
    path = str(tmp_path / "decode_tiny.qwb")
    mvb.qwb.write_synthetic_qwb(path, mvb.qwb.QWEN_TINY, seed=int(z["seed"]))
    dec = mvb.QwenDecoder(path, ctx=int(z["ctx"]))
    try:
        prompt, ids = [int(t) for t in z["prompt"]], [int(t) for t in z["ids"]]
        seq = prompt + ids
        logits = np.stack([dec.forward(seq[p], p)[1] for p in range(z["logits"].shape[0])])
        compare_logits(logits, z["logits"])
        got = dec.generate(prompt, len(ids))
        assert got.tolist() == ids
    finally:
        dec.close()


@pytest.fixture(scope="module")
def qwen05b(data_dir):
    mvb = load_pkg()
    path = mvb.qwb.cached_qwb(data_dir, mvb.qwb.QWEN05B, seed=0)
    dec = mvb.QwenDecoder(path, ctx=512)
    yield path, dec
    dec.close()


def test_qwen05b_logits_every_position(qwen05b, tmp_path):
    """16 prompt tokens + 16 greedy tokens: logits at all 31 positions against qwen.c's --logits dump."""
    path, dec = qwen05b
    prompt = [int(t) for t in np.random.default_rng(21).integers(0, 151936, 16)]
    ids = ref_run(path, prompt, 16, 512, str(tmp_path / "ref.bin"))
    ref = np.fromfile(tmp_path / "ref.bin", np.float32).reshape(-1, 65536)
    seq = prompt + ids
    ours = np.stack([dec.forward(seq[p], p)[1] for p in range(ref.shape[0])])
    compare_logits(ours, ref)
    assert dec.generate(prompt, 16).tolist() == ids


def test_qwen05b_full_run_ids(qwen05b):
    """The benchmark workload (config 3): 128 seeded prompt ids, 128 greedy tokens; identical ids to qwen.c."""
    path, dec = qwen05b
    prompt = [int(t) for t in np.random.default_rng(3).integers(0, 151936, 128)]
    r = subprocess.run([os.path.join(REF, "qwen"), path, "--ids", ",".join(map(str, prompt)), "-t", "0", "-n", "128",
                        "-c", "512"], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr
    ref_ids = [int(t) for t in r.stdout.strip().split(",") if t]
    got = dec.generate(prompt, 128).tolist()
    print("first ids", got[:12])
    assert got == ref_ids


def test_prefill_decode_equals_generate(qwen05b):
    """prefill + decode in pieces gives the same ids as one generate, and a rewound decode repeats itself."""
    _, dec = qwen05b
    prompt = [int(t) for t in np.random.default_rng(5).integers(0, 151936, 20)]
    whole = dec.generate(prompt, 24).tolist()
    dec.prefill(prompt)
    parts = dec.decode(10).tolist() + dec.decode(14).tolist()
    assert parts == whole
    dec.rewind(prompt[-1], len(prompt) - 1, len(prompt))
    assert dec.decode(24).tolist() == whole


@pytest.mark.parametrize("n", [1, 2, 37, 129, 300, 400])
def test_batched_prefill_equals_tokenwise(qwen05b, n):
    """The batched prefill (tensor-core matmuls, batched attention; batches of 256, so 300 tokens take two) writes
    the KV-cache rows of one decode step per token bit for bit, and decoding continues identically. At 400 tokens
    the second batch reaches 399 positions, more than the grouped attention stages in shared memory, so it runs the
    chunked one-CTA-per-query-head attention and the separate quantize."""
    _, dec = qwen05b
    prompt = [int(t) for t in np.random.default_rng(100 + n).integers(0, 151936, n)]
    dec.prefill_tokenwise(prompt)
    k_ref, v_ref = dec.cache(max(n - 1, 1))
    ids_ref = dec.decode(8).tolist()
    dec.prefill(prompt)
    k, v = dec.cache(max(n - 1, 1))
    if n > 1:
        assert np.array_equal(k.view(np.uint32), k_ref.view(np.uint32))
        assert np.array_equal(v.view(np.uint32), v_ref.view(np.uint32))
    assert dec.decode(8).tolist() == ids_ref


def test_tiny_batched_prefill_equals_tokenwise(tmp_path):
    mvb = load_pkg()
    path = str(tmp_path / "decode_tiny_batched.qwb")
    mvb.qwb.write_synthetic_qwb(path, mvb.qwb.QWEN_TINY, seed=11)
    dec = mvb.QwenDecoder(path, ctx=64)
    try:
        prompt = [int(t) for t in np.random.default_rng(4).integers(0, 1000, 40)]
        dec.prefill_tokenwise(prompt)
        k_ref, v_ref = dec.cache(39)
        ids_ref = dec.decode(6).tolist()
        dec.prefill(prompt)
        k, v = dec.cache(39)
        assert np.array_equal(k.view(np.uint32), k_ref.view(np.uint32))
        assert np.array_equal(v.view(np.uint32), v_ref.view(np.uint32))
        assert dec.decode(6).tolist() == ids_ref
    finally:
        dec.close()


def test_full_vocabulary_head(tmp_path):
    """mvb_qwen_full_head: the tied Q8 embedding as a vocab_size-row head. Its logits at the head_ids rows equal the
    trimmed head's bit for bit, its greedy row is the first maximum over the whole vocabulary (a token id), and
    switching back restores qwen.c's head."""
    mvb = load_pkg()
    path = str(tmp_path / "full_head.qwb")
    mvb.qwb.write_synthetic_qwb(path, mvb.qwb.QWEN_TINY, seed=17)
    head_ids = np.array(mvb.qwb.Qwb(path).head_ids)
    dec = mvb.QwenDecoder(path, ctx=64)
    try:
        vocab, hk = dec.cfg["vocab_size"], dec.cfg["head_k"]
        toks = [int(t) for t in np.random.default_rng(9).integers(0, vocab, 12)]
        for pos, tok in enumerate(toks):
            row_t, lt = dec.forward(tok, pos)
            dec.full_head(True)
            assert dec.cfg["head_k"] == vocab
            row_f, lf = dec.forward(tok, pos)
            assert lf.shape == (vocab,)
            assert np.array_equal(lf[head_ids].view(np.uint32), lt.view(np.uint32))
            assert row_f == int(np.argmax(lf))
            dec.full_head(False)
            assert dec.cfg["head_k"] == hk
            assert row_t == int(np.argmax(lt))
        # a whole greedy run over the full vocabulary: each id is the argmax of its position's full logits
        prompt = toks[:5]
        dec.full_head(True)
        ids = dec.generate(prompt, 10).tolist()
        seq = prompt + ids
        for p in range(len(prompt) - 1, len(seq) - 1):
            assert dec.forward(seq[p], p)[0] == seq[p + 1]
    finally:
        dec.close()


def test_load_rejects_bad_images(tmp_path):
    mvb = load_pkg()
    with pytest.raises(mvb.MatvecError):
        mvb.QwenDecoder(b"QWB2" + b"\0" * 300)
    path = str(tmp_path / "tiny.qwb")
    mvb.qwb.write_synthetic_qwb(path, mvb.qwb.QWEN_TINY, seed=11)
    bad = bytearray(open(path, "rb").read())
    with pytest.raises(mvb.MatvecError):
        mvb.QwenDecoder(bytes(bad[:-64]))  # size does not match the header (qwen.c:259-262)


def test_qwen05b_blocks_bit_exact_at_pos0(qwen05b):
    """Block-level parity on the full model: the device's residual stream after every attention and FFN block,
    against the same block computed on the CPU from the device's own block input with qwen.c's rmsnorm,
    quantize and matmul_cpu (oracle/_ref/libref_qwen.so). At position 0 attention returns v exactly (one
    position, softmax weight exp(0)/exp(0) = 1), and SiLU's expf is taken correctly rounded on both sides, so
    every block must agree bit for bit."""
    import oracle
    path, dec = qwen05b
    mvb = load_pkg()
    M = mvb.qwb.Qwb(path)
    rq = oracle.RefQwen()
    c = M.cfg
    dim, hid, L, eps = c["dim"], c["hidden_dim"], c["n_layers"], np.float32(c["rms_eps"])
    kv, hs = M.kv_dim, dim // c["n_heads"]
    kv_mul = c["n_heads"] // c["n_kv_heads"]
    tok = 4242
    tr = dec.trace(tok, 0)
    f16 = golden("f16_table.npz")["f32"]
    er, es = M.emb
    x0 = er[tok].view(np.int8).astype(np.float32) * f16[np.repeat(es[tok], 32)]
    assert np.array_equal(tr[0].view(np.uint32), x0.view(np.uint32))
    mm = lambda m, xq, xs, n, d: rq.matmul_cpu(m[0], m[1], xq, xs, n, d, 4)
    for l in range(L):
        x = tr[2 * l]
        xq, xs = rq.quantize(rq.rmsnorm(x, M.attn_norm[l], eps))
        v = mm(M.mats["wv"][l], xq, xs, dim, kv) + M.bv[l]
        att = np.float32(0) + np.repeat(v.reshape(-1, hs), kv_mul, axis=0).reshape(-1) * np.float32(1)
        q2, s2 = rq.quantize(att)
        x1 = x + mm(M.mats["wo"][l], q2, s2, dim, dim)
        assert np.array_equal(tr[2 * l + 1].view(np.uint32), x1.view(np.uint32)), f"attention block {l}"
        xq, xs = rq.quantize(rq.rmsnorm(tr[2 * l + 1], M.ffn_norm[l], eps))
        g = mm(M.mats["w1"][l], xq, xs, dim, hid)
        u = mm(M.mats["w3"][l], xq, xs, dim, hid)
        e = np.exp(-g.astype(np.float64)).astype(np.float32)
        hb = (g * (np.float32(1) / (np.float32(1) + e))) * u
        q3, s3 = rq.quantize(hb)
        x2 = tr[2 * l + 1] + mm(M.mats["w2"][l], q3, s3, hid, dim)
        assert np.array_equal(tr[2 * l + 2].view(np.uint32), x2.view(np.uint32)), f"ffn block {l}"


def test_step_stamps_partition_the_step(tmp_path):
    """mvb_qwen_stamps: one step as the graph runs it, every kernel stamping the global timer. Each kernel's first
    CTA gets past its wait no earlier than the previous kernel's last CTA ends (the programmatic dependency), every
    kernel ends after it starts, and the stamped step leaves the cache as a plain step would."""
    import torch
    mvb = load_pkg()
    z = golden("qwen_tiny.npz")
    path = str(tmp_path / "stamps_tiny.qwb")
    mvb.qwb.write_synthetic_qwb(path, mvb.qwb.QWEN_TINY, seed=int(z["seed"]))
    dec = mvb.QwenDecoder(path, ctx=64)
    try:
        seq = [int(t) for t in z["prompt"]] + [int(t) for t in z["ids"]]
        row_plain, _ = dec.forward(seq[0], 0)
        dec.rewind(seq[0], 0, -1)
        st = dec.stamps()
        assert st.shape == (dec.cfg["kernels_per_step"], 2)
        assert st[0, 0] == 0.0  # times are relative to the first kernel's start
        assert np.all(st[:, 1] >= st[:, 0])
        assert np.all(st[1:, 0] >= st[:-1, 1] - 0.05)  # 50 ns of timer granularity
        assert st[-1, 1] < 1e4  # a tiny model's step takes well under 10 ms
        # the stamped step is the same step: a plain step repeated after it picks the same head row
        dec.rewind(seq[0], 0, -1)
        row_again, _ = dec.forward(seq[0], 0)
        assert row_again == row_plain
    finally:
        dec.close()
