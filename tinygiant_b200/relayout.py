"""The reference's expert-contiguous on-disk format (tinygiant/relayout.py:142-157,
276-330; read by tinygiant/cache.py:32-57), for the B200 path.

A relayout directory holds one file per MoE layer, `layer_{L:03d}.q4.bin`: the layer's
experts in id order, each the raw bytes of its gate | up | down matrices (row-major by
output row, blocks contiguous per row).  `index.json` describes it:

    magic "NWSMOE01"; version (2 = the reference's Q4_K / Q6_K relayout, 3 = Q4_0 ggml
    blocks, 4 = Q4_0 in the row-split layout); dtype ("q4_k" or "q4_0"); layout ("ggml"
    or "rows", versions 3 / 4); n_layers, n_experts, n_experts_used, embed_dim;
    layers[L] = {file, total_bytes, expert_offsets[e] = {offset, sizes{gate, up, down}},
                 tensor_formats{gate, up, down}};
    q4_sizes{gate, up, down} = {out_dim, in_dim}; expert_shapes; activation_profile[L] =
    {expert_ranking, activation_counts} (optional)

The writer emits version 3 (ggml Q4_0 blocks) or, with layout="rows", version 4: every
matrix row as its blocks' 16-byte nibble groups followed by their fp16 scales, the
layout the device kernels read, so loads (tgx_load_experts_rows) and host-tier misses
copy the bytes as they are, with no repack.  The reader takes versions 2 to 4.  Layers
are read with pread straight into pinned host memory for the host tier (HostTierCache)
or copied into a device context.
"""
from __future__ import annotations

import json
import mmap
import os
from pathlib import Path

import numpy as np

from . import _constants as C

MAGIC = "NWSMOE01"
VERSION_Q4_0 = 3
VERSION_Q4_0_ROWS = 4
LAYOUT_GGML, LAYOUT_ROWS = "ggml", "rows"
EXPERT_KEYS = C.EXPERT_KEYS_ORDER          # gate, up, down


def layer_file_name(layer: int) -> str:
    return f"layer_{layer:03d}.q4.bin"


def q4_0_matrix_bytes(out_dim: int, in_dim: int) -> int:
    return out_dim * (in_dim // C.QK) * C.Q4_0_BYTES


def rows_from_ggml(blocks: np.ndarray, nrows: int, nb: int) -> np.ndarray:
    """Q4_0 rows of nb ggml blocks (fp16 d | 16 nibble bytes, 18 B each) -> row-split rows:
    the nb 16-byte nibble groups, then the nb fp16 scales (same bytes per row)."""
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(nrows, nb, C.Q4_0_BYTES)
    out = np.empty((nrows, nb * C.Q4_0_BYTES), np.uint8)
    out[:, :nb * 16] = b[:, :, 2:].reshape(nrows, nb * 16)
    out[:, nb * 16:] = b[:, :, :2].reshape(nrows, nb * 2)
    return out.reshape(-1)


def ggml_from_rows(rows: np.ndarray, nrows: int, nb: int) -> np.ndarray:
    """The inverse of rows_from_ggml."""
    r = np.ascontiguousarray(rows, dtype=np.uint8).reshape(nrows, nb * C.Q4_0_BYTES)
    out = np.empty((nrows, nb, C.Q4_0_BYTES), np.uint8)
    out[:, :, 2:] = r[:, :nb * 16].reshape(nrows, nb, 16)
    out[:, :, :2] = r[:, nb * 16:].reshape(nrows, nb, 2)
    return out.reshape(-1)


def _expert_matrices(embed: int, inter: int):
    """(rows, blocks per row) of gate, up, down."""
    return ((inter, embed // C.QK), (inter, embed // C.QK), (embed, inter // C.QK))


def expert_convert(blob: np.ndarray, embed: int, inter: int, to_rows: bool) -> np.ndarray:
    """One expert blob gate | up | down between the ggml and row-split layouts."""
    blob = np.ascontiguousarray(blob, dtype=np.uint8)
    parts, pos = [], 0
    for rows, nb in _expert_matrices(embed, inter):
        n = rows * nb * C.Q4_0_BYTES
        fn = rows_from_ggml if to_rows else ggml_from_rows
        parts.append(fn(blob[pos:pos + n], rows, nb))
        pos += n
    assert pos == blob.size
    return np.concatenate(parts)


def write_layer(out_dir, layer: int, experts, formats=None) -> dict:
    """Write one layer file: experts[e] = (gate, up, down) byte arrays, in id order
    (the reference's write_expert_cache_q4, relayout.py:142-157).  Returns the layer's
    index entry."""
    out_dir = Path(out_dir)
    offsets, pos = {}, 0
    with open(out_dir / layer_file_name(layer), "wb") as f:
        for e, parts in enumerate(experts):
            sizes = {}
            start = pos
            for key, data in zip(EXPERT_KEYS, parts):
                b = np.ascontiguousarray(data).view(np.uint8)
                f.write(b.tobytes())
                sizes[key] = int(b.nbytes)
                pos += b.nbytes
            offsets[str(e)] = {"offset": start, "sizes": sizes}
    return {"file": layer_file_name(layer), "total_bytes": pos, "expert_offsets": offsets,
            "tensor_formats": dict(formats or {k: "q4_0" for k in EXPERT_KEYS})}


def write_index(out_dir, layers: dict, n_experts: int, n_experts_used: int, embed_dim: int, inter_dim: int,
                n_layers: int | None = None, activation_profile=None, model: str = "synthetic",
                layout: str = LAYOUT_GGML) -> dict:
    """index.json for a Q4_0 relayout (the reference's fields, relayout.py:276-330, with
    dtype "q4_0" and version 3, or version 4 with layout "rows")."""
    assert layout in (LAYOUT_GGML, LAYOUT_ROWS)
    index = {
        "magic": MAGIC, "version": VERSION_Q4_0_ROWS if layout == LAYOUT_ROWS else VERSION_Q4_0,
        "layout": layout, "model": model,
        "n_layers": n_layers if n_layers is not None else len(layers), "n_experts": n_experts,
        "n_experts_used": n_experts_used, "embed_dim": embed_dim, "dtype": "q4_0",
        "expert_shapes": {"gate": [inter_dim, embed_dim], "up": [inter_dim, embed_dim], "down": [embed_dim, inter_dim]},
        "q4_sizes": {"gate": {"out_dim": inter_dim, "in_dim": embed_dim},
                     "up": {"out_dim": inter_dim, "in_dim": embed_dim},
                     "down": {"out_dim": embed_dim, "in_dim": inter_dim}},
        "tensor_formats": {k: "q4_0" for k in EXPERT_KEYS},
        "layers": {str(k): v for k, v in layers.items()},
        "activation_profile": activation_profile or {},
    }
    with open(Path(out_dir) / "index.json", "w") as f:
        json.dump(index, f, indent=2)
    return index


def write_model(out_dir, layer_blobs, n_experts: int, n_experts_used: int, embed_dim: int, inter_dim: int,
                activation_profile=None, layout: str = LAYOUT_GGML) -> dict:
    """A whole Q4_0 relayout from per-layer blobs (E experts, each gate | up | down,
    ggml Q4_0, expert-contiguous, as tgx_read_experts returns them); layout "rows"
    stores every expert in the row-split layout (version 4)."""
    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    gb = q4_0_matrix_bytes(inter_dim, embed_dim)
    db = q4_0_matrix_bytes(embed_dim, inter_dim)
    eb = 2 * gb + db
    layers = {}
    for l, blob in enumerate(layer_blobs):
        blob = np.ascontiguousarray(blob, dtype=np.uint8)
        assert blob.size == n_experts * eb
        experts = []
        for e in range(n_experts):
            x = blob[e * eb:(e + 1) * eb]
            if layout == LAYOUT_ROWS:
                x = expert_convert(x, embed_dim, inter_dim, True)
            experts.append((x[:gb], x[gb:2 * gb], x[2 * gb:]))
        fmt = "q4_0_rows" if layout == LAYOUT_ROWS else "q4_0"
        layers[l] = write_layer(out_dir, l, experts, {k: fmt for k in EXPERT_KEYS})
    return write_index(out_dir, layers, n_experts, n_experts_used, embed_dim, inter_dim, len(layer_blobs),
                       activation_profile, layout=layout)


SUPPORTED_VERSIONS = (2, VERSION_Q4_0, VERSION_Q4_0_ROWS)


class RelayoutReader:
    """Reads a relayout directory: version 2 (the reference's writer, Q4_K / Q6_K / f16
    experts), 3 (Q4_0 ggml blocks) or 4 (Q4_0 in the kernels' row-split rows).  Any other
    version is rejected, since its byte layout is unknown."""

    def __init__(self, path):
        self.dir = Path(path)
        with open(self.dir / "index.json") as f:
            self.index = json.load(f)
        if self.index.get("magic") != MAGIC:
            raise ValueError(f"{self.dir}: not a relayout index (magic {self.index.get('magic')!r})")
        self.version = int(self.index.get("version", 0))
        if self.version not in SUPPORTED_VERSIONS:
            raise ValueError(f"{self.dir}: relayout version {self.version} is not one of {SUPPORTED_VERSIONS}")
        self.dtype = self.index.get("dtype")
        self.layout = self.index.get("layout", LAYOUT_ROWS if self.version == VERSION_Q4_0_ROWS else LAYOUT_GGML)
        self.layers = {int(k): v for k, v in self.index["layers"].items()}
        self.n_experts = int(self.index["n_experts"])
        self._maps = {}

    def formats(self, layer: int) -> dict:
        fmt = self.layers[layer].get("tensor_formats") or self.index.get("tensor_formats") or {}
        default = "q4_0" if self.dtype == "q4_0" else "q4_k"
        return {k: fmt.get(k, default) for k in EXPERT_KEYS}

    def path(self, layer: int) -> Path:
        return self.dir / self.layers[layer]["file"]

    def _map(self, layer: int):
        if layer not in self._maps:
            f = open(self.path(layer), "rb")
            self._maps[layer] = (f, mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ))
        return self._maps[layer][1]

    def expert(self, layer: int, e: int) -> dict:
        """{gate, up, down}: read-only uint8 views of one expert's matrices (cache.py:42-57)."""
        info = self.layers[layer]["expert_offsets"][str(e)]
        mm, pos, out = self._map(layer), int(info["offset"]), {}
        for k in EXPERT_KEYS:
            n = int(info["sizes"][k])
            out[k] = np.frombuffer(mm, dtype=np.uint8, count=n, offset=pos)
            pos += n
        return out

    def expert_ggml(self, layer: int, e: int) -> np.ndarray:
        """One Q4_0 expert as a ggml blob, whatever the file's layout."""
        blob = self.expert_blob(layer, e)
        if self.layout != LAYOUT_ROWS:
            return blob
        return expert_convert(blob, int(self.index["embed_dim"]), int(self.index["q4_sizes"]["gate"]["out_dim"]),
                              False)

    def expert_blob(self, layer: int, e: int) -> np.ndarray:
        info = self.layers[layer]["expert_offsets"][str(e)]
        n = sum(int(info["sizes"][k]) for k in EXPERT_KEYS)
        return np.frombuffer(self._map(layer), dtype=np.uint8, count=n, offset=int(info["offset"]))

    def layer_bytes(self, layer: int) -> np.ndarray:
        """The whole layer file (experts in id order, contiguous) as a read-only view."""
        return np.frombuffer(self._map(layer), dtype=np.uint8, count=int(self.layers[layer]["total_bytes"]))

    def read_layer_into(self, layer: int, dst: np.ndarray, chunk: int = 64 << 20) -> None:
        """pread the layer file into dst (any writable uint8 buffer, e.g. pinned host memory)."""
        n = int(self.layers[layer]["total_bytes"])
        assert dst.dtype == np.uint8 and dst.size >= n
        fd = os.open(self.path(layer), os.O_RDONLY)
        try:
            view = memoryview(dst)
            done = 0
            while done < n:
                got = os.preadv(fd, [view[done:min(n, done + chunk)]], done)
                if got <= 0:
                    raise OSError(f"{self.path(layer)}: short read at {done} of {n}")
                done += got
        finally:
            os.close(fd)

    def read_layer_pinned(self, layer: int):
        """The layer file in pinned host memory (a torch uint8 tensor), for HostTierCache."""
        import torch
        n = int(self.layers[layer]["total_bytes"])
        t = torch.empty(n, dtype=torch.uint8, pin_memory=True)
        self.read_layer_into(layer, t.numpy())
        return t

    def hot_experts(self, layer: int, n: int):
        """The profile's most active experts of a layer (cache.py:84-100's ranking)."""
        prof = (self.index.get("activation_profile") or {}).get(str(layer))
        return list(prof["expert_ranking"][:n]) if prof else []

    def load_into(self, model) -> None:
        """Copy every layer into an engine.MoEModel (Q4_0 relayouts only); a "rows" file
        goes in as it is, a ggml one through the device repack."""
        if self.dtype != "q4_0":
            raise ValueError(f"load_into needs a q4_0 relayout, not {self.dtype!r}")
        for layer in sorted(self.layers):
            if self.layout == LAYOUT_ROWS:
                model.load_experts_rows(layer, self.layer_bytes(layer))
            else:
                model.load_experts(layer, self.layer_bytes(layer))

    def close(self):
        """Drop the mappings; one still viewed by an array handed out stays mapped until
        that array is gone."""
        for f, mm in self._maps.values():
            try:
                mm.close()
            except BufferError:
                pass
            f.close()
        self._maps.clear()
