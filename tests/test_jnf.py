"""JNF v1 expert store (tarfa_b200/jnf.py) on CPU.

The reader follows the reference's format rules (format/JNF_V1.md; the layout
format/convert_jnf.py:53-86 writes): every expert projection read back is bit
for bit what was written; a changed byte fails its SHA-256; unknown versions,
dtypes, shapes, unaligned projections, wrong offsets and truncated files are
refused when the store is opened; writes are atomic (no ``.partial`` left)."""
import json
import os

import pytest
import torch

from tarfa_b200 import jnf

E, I, H = 8, 64, 128   # gate_up expert 32 KiB, down expert 16 KiB: both 4096-aligned


def _layer(seed):
    g = torch.Generator().manual_seed(seed)
    gu = (torch.randn((E, 2 * I, H), generator=g) * 0.02).to(torch.bfloat16)
    dn = (torch.randn((E, H, I), generator=g) * 0.02).to(torch.bfloat16)
    return gu, dn


@pytest.fixture
def store(tmp_path):
    layers = {l: _layer(l) for l in (0, 3)}
    for l, (gu, dn) in layers.items():
        jnf.write_layer(tmp_path, l, gu, dn)
    return tmp_path, layers


def test_round_trip_bit_exact(store):
    root, layers = store
    s = jnf.JnfStore(root)
    assert s.layers == [0, 3]
    assert s.dims(3) == (E, I, H)
    for l, (gu, dn) in layers.items():
        rgu, rdn = s.read_layer(l, pin=False)
        assert torch.equal(rgu.view(torch.int16), gu.view(torch.int16))
        assert torch.equal(rdn.view(torch.int16), dn.view(torch.int16))
        sub = [5, 1, 6]
        sgu, sdn = s.read_experts(l, sub, pin=False)
        assert torch.equal(sgu.view(torch.int16), gu[sub].view(torch.int16))
        assert torch.equal(sdn.view(torch.int16), dn[sub].view(torch.int16))
        s.verify_layer(l)
    m = json.loads((root / "manifest.json").read_text())
    assert (m["format"], m["version"], m["dtype"], m["alignment"]) == ("JNF", 1, "BF16", 4096)
    ix = json.loads((root / "layers" / "03" / "index.json").read_text())
    assert ix["gate_up"]["offsets"] == [e * 2 * I * H * 2 for e in range(E)]
    assert not list(root.rglob("*.partial"))


def test_changed_byte_fails_its_hash(store):
    root, _ = store
    f = root / "layers" / "00" / "down.bf16"
    b = bytearray(f.read_bytes())
    b[3 * H * I * 2 + 17] ^= 0x01          # expert 3
    f.write_bytes(bytes(b))
    s = jnf.JnfStore(root)
    s.read_experts(0, [0, 1, 2], pin=False)                    # other experts still read
    with pytest.raises(jnf.JnfError, match="expert 3: SHA-256"):
        s.read_experts(0, [3], pin=False)
    with pytest.raises(jnf.JnfError, match="SHA-256"):
        s.verify_layer(0)
    jnf.JnfStore(root, verify=False).read_experts(0, [3], pin=False)


def _edit_manifest(root, fn):
    p = root / "manifest.json"
    m = json.loads(p.read_text())
    fn(m)
    p.write_text(json.dumps(m))


@pytest.mark.parametrize("edit,msg", [
    (lambda m: m.update(version=2), "version"),
    (lambda m: m.update(format="XYZ"), "format"),
    (lambda m: m.update(dtype="F16"), "dtype"),
    (lambda m: m["layers"]["0"]["down_proj"].update(shape=[E, H, I + 1]), "expert_bytes"),
    (lambda m: m["layers"]["0"]["gate_up_proj"]["expert_sha256"].pop(), "hashes"),
    (lambda m: m["layers"]["0"]["down_proj"].update(shape=[E, H * 2, I // 2]), "one expert layout"),
])
def test_refused_manifests(store, edit, msg):
    root, _ = store
    _edit_manifest(root, edit)
    with pytest.raises(jnf.JnfError, match=msg):
        jnf.JnfStore(root)


def test_truncated_file_and_bad_offsets_refused(store):
    root, _ = store
    ix = root / "layers" / "03" / "index.json"
    d = json.loads(ix.read_text())
    d["down"]["offsets"][2] += 4096
    ix.write_text(json.dumps(d))
    with pytest.raises(jnf.JnfError, match="offsets"):
        jnf.JnfStore(root)
    f = root / "layers" / "00" / "gate_up.bf16"
    with open(f, "r+b") as fh:
        fh.truncate(os.path.getsize(f) - 4096)
    with pytest.raises(jnf.JnfError, match="holds"):
        jnf.JnfStore(root)


def test_unaligned_projection_refused_on_write(tmp_path):
    gu = torch.zeros((2, 2 * 8, 24), dtype=torch.bfloat16)    # 768-byte experts
    dn = torch.zeros((2, 24, 8), dtype=torch.bfloat16)
    with pytest.raises(jnf.JnfError, match="4096"):
        jnf.write_layer(tmp_path, 0, gu, dn)
