"""JNF v1 expert store: the reference's on-disk execution format, read (and written).

Layout (the reference's ``format/JNF_V1.md``; written by
``format/convert_jnf.py:53-86``)::

    <root>/manifest.json            format "JNF", version 1, dtype "BF16",
                                    alignment 4096, router_top_k, model and
                                    tokenizer revisions, and per layer:
        layers["<l>"]["gate_up_proj" | "down_proj"] =
            {file, shape [E, N, K], expert_bytes, file_sha256, expert_sha256[E]}
    <root>/layers/<ll>/gate_up.bf16  expert e's [2I, H] projection at byte e * expert_bytes
    <root>/layers/<ll>/down.bf16     expert e's [H, I] projection likewise
    <root>/layers/<ll>/index.json    the per-expert byte offsets

Every rule the format states is checked when a store is opened, and the
reader refuses the store (``JnfError``) otherwise:
- the format name and version 1;
- BF16;
- ``expert_bytes`` equal to the shape's bytes and a multiple of the 4096-byte alignment;
- offsets ``e * expert_bytes``;
- file sizes ``E * expert_bytes``;
- gate_up ``[E, 2I, H]`` against down ``[E, H, I]``.

SHA-256 of every expert projection read is checked against the manifest
(``verify=True``, the default); :meth:`JnfStore.verify_layer` re-hashes whole
files.  Reads go straight into the caller's (pinned) host tensors with
``os.preadv``: no intermediate copy.  The streaming tier
(``StreamingExpertTier.load_layer_jnf``) places a layer from a store.

:func:`write_layer` writes a layer the same way the reference's converter
does, atomically (``.partial`` then rename).  It is for the tests and for
users who convert their own weights.
"""
from __future__ import annotations

import hashlib
import json
import os
from pathlib import Path

import torch

FORMAT, VERSION, ALIGN = "JNF", 1, 4096
_PROJ = {"gate_up_proj": "gate_up.bf16", "down_proj": "down.bf16"}


class JnfError(RuntimeError):
    pass


def _pread_into(fd: int, offset: int, buf: memoryview) -> None:
    done = 0
    while done < len(buf):
        n = os.preadv(fd, [buf[done:]], offset + done)
        if n <= 0:
            raise JnfError(f"short read at byte {offset + done}")
        done += n


def _bytes_view(t: torch.Tensor) -> memoryview:
    if t.device.type != "cpu" or not t.is_contiguous() or t.dtype != torch.bfloat16:
        raise JnfError("JNF reads go into contiguous bf16 host tensors")
    return memoryview(t.view(torch.uint8).numpy()).cast("B")


class JnfStore:
    """A JNF v1 tree opened for reading; the manifest is validated up front."""

    def __init__(self, root, verify: bool = True):
        self.root = Path(root)
        self.verify = verify
        mpath = self.root / "manifest.json"
        if not mpath.exists():
            raise JnfError(f"{mpath}: no manifest")
        m = json.loads(mpath.read_text())
        if m.get("format") != FORMAT or m.get("version") != VERSION:
            raise JnfError(f"unknown store format {m.get('format')!r} version {m.get('version')!r}")
        if m.get("dtype") != "BF16":
            raise JnfError(f"dtype {m.get('dtype')!r} (JNF v1 is BF16)")
        if m.get("alignment", ALIGN) != ALIGN:
            raise JnfError(f"alignment {m.get('alignment')} (JNF v1 is {ALIGN})")
        self.manifest = m
        self.top_k = int(m.get("router_top_k", 8))
        self._layers = {int(k): v for k, v in m.get("layers", {}).items()}
        self._dims = {}
        for l, rec in self._layers.items():
            self._dims[l] = self._check_layer(l, rec)

    # -- validation ----------------------------------------------------------------
    def _check_layer(self, l, rec):
        for name in _PROJ:
            if name not in rec:
                raise JnfError(f"layer {l}: no {name}")
            r = rec[name]
            shape = [int(x) for x in r["shape"]]
            if len(shape) != 3:
                raise JnfError(f"layer {l} {name}: shape {shape}")
            eb = int(r["expert_bytes"])
            if eb != shape[1] * shape[2] * 2:
                raise JnfError(f"layer {l} {name}: expert_bytes {eb} != shape {shape} in BF16")
            if eb % ALIGN:
                raise JnfError(f"layer {l} {name}: expert_bytes {eb} not a multiple of {ALIGN}")
            if len(r["expert_sha256"]) != shape[0]:
                raise JnfError(f"layer {l} {name}: {len(r['expert_sha256'])} expert hashes, {shape[0]} experts")
            path = self.root / r["file"]
            if not path.exists():
                raise JnfError(f"layer {l} {name}: {path} missing")
            if path.stat().st_size != shape[0] * eb:
                raise JnfError(f"layer {l} {name}: {path} holds {path.stat().st_size} bytes, "
                               f"expected {shape[0] * eb}")
        gu, dn = rec["gate_up_proj"]["shape"], rec["down_proj"]["shape"]
        E, I2, H = gu
        if I2 % 2 or dn != [E, H, I2 // 2]:
            raise JnfError(f"layer {l}: gate_up {gu} and down {dn} do not form one expert layout")
        idx = self.root / "layers" / f"{l:02d}" / "index.json"
        if idx.exists():
            ix = json.loads(idx.read_text())
            for key, name in (("gate_up", "gate_up_proj"), ("down", "down_proj")):
                eb = rec[name]["expert_bytes"]
                if ix[key]["offsets"] != [e * eb for e in range(E)]:
                    raise JnfError(f"layer {l} {key}: index offsets are not e * {eb}")
        return E, I2 // 2, H

    # -- queries -------------------------------------------------------------------
    @property
    def layers(self):
        return sorted(self._layers)

    def dims(self, layer: int):
        """(E, I, H) of a layer."""
        if layer not in self._dims:
            raise JnfError(f"layer {layer} not in the store")
        return self._dims[layer]

    # -- reads ---------------------------------------------------------------------
    def _read(self, layer, name, experts, out: torch.Tensor):
        r = self._layers[layer][name]
        eb = int(r["expert_bytes"])
        view = _bytes_view(out)
        if len(view) != len(experts) * eb:
            raise JnfError(f"output holds {len(view)} bytes, {len(experts)} experts need {len(experts) * eb}")
        fd = os.open(self.root / r["file"], os.O_RDONLY)
        try:
            for j, e in enumerate(experts):
                if not 0 <= e < len(r["expert_sha256"]):
                    raise JnfError(f"expert {e} out of range")
                part = view[j * eb:(j + 1) * eb]
                _pread_into(fd, e * eb, part)
                if self.verify and hashlib.sha256(part).hexdigest() != r["expert_sha256"][e]:
                    raise JnfError(f"layer {layer} {name} expert {e}: SHA-256 mismatch")
        finally:
            os.close(fd)

    def read_experts(self, layer: int, experts, gate_up: torch.Tensor | None = None,
                     down: torch.Tensor | None = None, pin: bool = True):
        """Experts ``experts`` of ``layer`` as ``gate_up [n, 2I, H]`` and ``down [n, H, I]``
        bf16 host tensors (pinned when allocated here; or the caller's tensors)."""
        E, I, H = self.dims(layer)
        experts = [int(e) for e in experts]
        n = len(experts)
        if gate_up is None:
            gate_up = torch.empty((n, 2 * I, H), dtype=torch.bfloat16, pin_memory=pin)
        if down is None:
            down = torch.empty((n, H, I), dtype=torch.bfloat16, pin_memory=pin)
        if tuple(gate_up.shape) != (n, 2 * I, H) or tuple(down.shape) != (n, H, I):
            raise JnfError("output shapes do not match the layer")
        self._read(layer, "gate_up_proj", experts, gate_up)
        self._read(layer, "down_proj", experts, down)
        return gate_up, down

    def read_layer(self, layer: int, pin: bool = True):
        E, _, _ = self.dims(layer)
        return self.read_experts(layer, range(E), pin=pin)

    def verify_layer(self, layer: int) -> None:
        """Re-hash both files of a layer, whole and per expert; raises on a mismatch."""
        self.dims(layer)
        for name in _PROJ:
            r = self._layers[layer][name]
            eb = int(r["expert_bytes"])
            whole = hashlib.sha256()
            with open(self.root / r["file"], "rb") as f:
                for e, want in enumerate(r["expert_sha256"]):
                    d = f.read(eb)
                    whole.update(d)
                    if hashlib.sha256(d).hexdigest() != want:
                        raise JnfError(f"layer {layer} {name} expert {e}: SHA-256 mismatch")
            if whole.hexdigest() != r["file_sha256"]:
                raise JnfError(f"layer {layer} {name}: file SHA-256 mismatch")


def write_layer(root, layer: int, gate_up: torch.Tensor, down: torch.Tensor,
                meta: dict | None = None) -> None:
    """Write one layer's experts (``gate_up [E, 2I, H]``, ``down [E, H, I]`` bf16) in
    JNF v1, each file as ``.partial`` then renamed, and add it to the manifest
    (rewritten the same way)."""
    root = Path(root)
    gate_up = gate_up.detach().to("cpu", torch.bfloat16).contiguous()
    down = down.detach().to("cpu", torch.bfloat16).contiguous()
    E, I2, H = gate_up.shape
    if tuple(down.shape) != (E, H, I2 // 2):
        raise JnfError("gate_up [E, 2I, H] and down [E, H, I] do not match")
    ld = root / "layers" / f"{layer:02d}"
    ld.mkdir(parents=True, exist_ok=True)
    rec, index = {}, {"layer": layer}
    for name, t in (("gate_up_proj", gate_up), ("down_proj", down)):
        eb = t[0].numel() * 2
        if eb % ALIGN:
            raise JnfError(f"{name}: expert bytes {eb} not a multiple of {ALIGN}")
        final = ld / _PROJ[name]
        partial = final.with_suffix(".partial")
        whole, hashes = hashlib.sha256(), []
        raw = t.view(torch.uint8).numpy()
        with open(partial, "wb") as f:
            for e in range(E):
                d = raw[e].tobytes()
                f.write(d)
                whole.update(d)
                hashes.append(hashlib.sha256(d).hexdigest())
        os.replace(partial, final)
        rec[name] = {"file": str(final.relative_to(root)), "shape": list(t.shape), "expert_bytes": eb,
                     "file_sha256": whole.hexdigest(), "expert_sha256": hashes}
        index["gate_up" if name == "gate_up_proj" else "down"] = {
            "expert_bytes": eb, "offsets": [e * eb for e in range(E)]}
    (ld / "index.json").write_text(json.dumps(index))
    mpath = root / "manifest.json"
    if mpath.exists():
        m = json.loads(mpath.read_text())
    else:
        m = {"format": FORMAT, "version": VERSION, "dtype": "BF16", "alignment": ALIGN,
             "router_top_k": 8, "model_id": None, "revision": None, "tokenizer_revision": None,
             "layers": {}}
        m.update(meta or {})
    m["layers"][str(layer)] = rec
    tmp = root / "manifest.json.partial"
    tmp.write_text(json.dumps(m, indent=1))
    os.replace(tmp, mpath)
