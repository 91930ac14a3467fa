"""GPU: `ane-lm convert` end to end through the C ABI -- safetensors files in,
ANE blob files out, byte-identical to the reference writer."""
import json
import os

import numpy as np
import pytest

from safetensors_util import blob_bytes, write_safetensors

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def read_tree(root):
    out = {}
    for d, _, files in os.walk(root):
        for f in files:
            p = os.path.join(d, f)
            out[os.path.relpath(p, root)] = open(p, "rb").read()
    return out


def test_golden_blobs_byte_identical(ane, tmp_path):
    g = np.load(os.path.join(GOLDEN, "convert_blobs.npz"))
    st = tmp_path / "model.safetensors"
    st.write_bytes(g["safetensors"].tobytes())
    out = tmp_path / "ane_weights"
    assert ane.write_ane_blobs(str(st), str(out)) == 3  # the F32 tensor is skipped
    tree = read_tree(out)
    for key in g.files:
        if key.startswith("blob:"):
            rel = key[5:].replace(".", "/") + ".bin"
            assert tree.pop(rel) == g[key].tobytes(), rel
    assert not tree


def test_sharded_model_dir(ane, oracle, tmp_path):
    rng = np.random.default_rng(0)
    md = tmp_path / "model"
    md.mkdir()
    big = rng.integers(0, 65536, size=(5, 7_000_003), dtype=np.uint16)  # > two 16 Mi chunks
    small = rng.integers(0, 65536, size=(64, 48), dtype=np.uint16)
    norm = rng.integers(0, 65536, size=(48,), dtype=np.uint16)
    shard1 = [("model.embed_tokens.weight", "BF16", big), ("model.norm.weight", "BF16", norm),
              ("model.layers.0.bias", "F16", rng.standard_normal(8).astype(np.float16))]
    shard2 = [("model.layers.0.mlp.up_proj.weight", "BF16", small),
              ("model.norm.weight", "BF16", small[:1, :48].ravel())]  # later shard wins
    write_safetensors(md / "model-00001-of-00002.safetensors", shard1)
    write_safetensors(md / "model-00002-of-00002.safetensors", shard2)
    wm = {n: "model-00001-of-00002.safetensors" for n, _, _ in shard1}
    wm.update({n: "model-00002-of-00002.safetensors" for n, _, _ in shard2})
    (md / "model.safetensors.index.json").write_text(json.dumps({"weight_map": wm}))
    out = tmp_path / "out"
    assert ane.convert_model(str(md), str(out)) == 4
    tree = read_tree(out)
    want = {
        "model/embed_tokens/weight.bin": blob_bytes(oracle.bf16_to_f16(big.ravel())),
        "model/layers/0/mlp/up_proj/weight.bin": blob_bytes(oracle.bf16_to_f16(small.ravel())),
        "model/norm/weight.bin": blob_bytes(oracle.bf16_to_f16(small[:1, :48].ravel())),
    }
    assert set(tree) == set(want)
    for k, v in want.items():
        assert tree[k] == v, k


def test_recursive_discovery_without_index(ane, oracle, tmp_path):
    rng = np.random.default_rng(1)
    md = tmp_path / "m"
    (md / "sub").mkdir(parents=True)
    a = rng.integers(0, 65536, size=(3, 5), dtype=np.uint16)
    b = rng.integers(0, 65536, size=(7,), dtype=np.uint16)
    write_safetensors(md / "b.safetensors", [("x.y", "BF16", a)])
    write_safetensors(md / "sub" / "a.safetensors", [("z", "BF16", b)])
    out = tmp_path / "o"
    assert ane.convert_model(str(md), str(out)) == 2
    tree = read_tree(out)
    assert tree["x/y.bin"] == blob_bytes(oracle.bf16_to_f16(a.ravel()))
    assert tree["z.bin"] == blob_bytes(oracle.bf16_to_f16(b))


def test_repeated_tensors_last_shard_wins(ane, oracle, tmp_path):
    """Tensors repeated across shards: the reference writes shards in order, so
    the last shard's data ends in the file, and every write is counted.  The
    conversion runs on several threads; the result must not depend on them."""
    rng = np.random.default_rng(3)
    md = tmp_path / "model"
    md.mkdir()
    names = [f"model.layers.{i}.self_attn.q_proj.weight" for i in range(6)]
    wm, last = {}, {}
    for sh in range(3):
        fn = f"model-{sh + 1:05d}-of-00003.safetensors"
        tensors = []
        for i, n in enumerate(names):
            a = rng.integers(0, 65536, size=(64, 1000 + 37 * i + sh), dtype=np.uint16)
            tensors.append((n, "BF16", a))
            last[n] = a
            wm[n] = fn
        write_safetensors(md / fn, tensors)
    (md / "model.safetensors.index.json").write_text(
        json.dumps({"weight_map": {f"t{i}": f"model-{i % 3 + 1:05d}-of-00003.safetensors"
                                   for i in range(3)}}))
    out = tmp_path / "out"
    for _ in range(2):  # the second run overwrites the same tree
        assert ane.convert_model(str(md), str(out)) == 18
        tree = read_tree(out)
        assert set(tree) == {n.replace(".", "/") + ".bin" for n in names}
        for n in names:
            assert tree[n.replace(".", "/") + ".bin"] == blob_bytes(oracle.bf16_to_f16(last[n].ravel())), n


def test_write_failure_in_a_worker_is_reported(ane, tmp_path):
    """A blob that cannot be created (its directory is a file) fails the call
    with the message of the thread that met it."""
    rng = np.random.default_rng(4)
    st = tmp_path / "model.safetensors"
    write_safetensors(st, [(f"w{i}.weight", "BF16", rng.integers(0, 65536, 5000, dtype=np.uint16))
                           for i in range(8)])
    out = tmp_path / "out"
    out.write_text("not a directory")
    with pytest.raises(ane.AneCudaError) as e:
        ane.write_ane_blobs(str(st), str(out))
    assert "cannot write" in str(e.value)
