"""The relayout format (tinygiant/relayout.py:142-157, 276-330; tinygiant/cache.py:32-57):
writer, reader, pread ingest, and the reference's own version-2 Q4_K / Q6_K indexes."""
from __future__ import annotations

import json

import numpy as np
import pytest

from tinygiant_b200 import relayout as R


def _blob(rng, n):
    return rng.integers(0, 256, size=n, dtype=np.uint8)


def test_write_and_read_q4_0_relayout(tmp_path):
    rng = np.random.default_rng(0)
    H, I, E, L = 256, 256, 4, 2
    eb = 3 * I * (H // 32) * 18
    blobs = [_blob(rng, E * eb) for _ in range(L)]
    prof = {"1": {"expert_ranking": [3, 1, 0, 2], "activation_counts": [5, 9, 1, 20]}}
    idx = R.write_model(tmp_path, blobs, E, 2, H, I, activation_profile=prof)
    assert idx["magic"] == "NWSMOE01" and idx["version"] == 3 and idx["dtype"] == "q4_0"
    on_disk = json.loads((tmp_path / "index.json").read_text())
    assert on_disk["layers"]["1"]["file"] == "layer_001.q4.bin"
    rd = R.RelayoutReader(tmp_path)
    gb = I * (H // 32) * 18
    for l in range(L):
        assert np.array_equal(rd.layer_bytes(l), blobs[l])
        assert rd.formats(l) == {"gate": "q4_0", "up": "q4_0", "down": "q4_0"}
        for e in range(E):
            ex = rd.expert(l, e)
            assert ex["gate"].size == gb and ex["down"].size == gb
            assert np.array_equal(np.concatenate([ex["gate"], ex["up"], ex["down"]]), blobs[l][e * eb:(e + 1) * eb])
            assert np.array_equal(rd.expert_blob(l, e), blobs[l][e * eb:(e + 1) * eb])
        dst = np.zeros(E * eb + 7, np.uint8)
        rd.read_layer_into(l, dst, chunk=1000)          # pread in small chunks
        assert np.array_equal(dst[:E * eb], blobs[l])
    assert rd.hot_experts(1, 2) == [3, 1] and rd.hot_experts(0, 2) == []
    rd.close()


def test_row_split_conversion():
    # rows of blocks: nibble groups first, then the fp16 scales; and back
    rng = np.random.default_rng(5)
    g = _blob(rng, 2 * 3 * 18)                       # 2 rows x 3 blocks
    r = R.rows_from_ggml(g, 2, 3)
    assert r.size == g.size
    b = g.reshape(2, 3, 18)
    assert np.array_equal(r.reshape(2, 54)[:, :48], b[:, :, 2:].reshape(2, 48))
    assert np.array_equal(r.reshape(2, 54)[:, 48:], b[:, :, :2].reshape(2, 6))
    assert np.array_equal(R.ggml_from_rows(r, 2, 3), g)
    H, I = 512, 256
    eb = 3 * I * (H // 32) * 18
    x = _blob(rng, eb)
    y = R.expert_convert(x, H, I, True)
    gb = I * (H // 32) * 18
    assert np.array_equal(y[:gb], R.rows_from_ggml(x[:gb], I, H // 32))               # gate
    assert np.array_equal(y[2 * gb:], R.rows_from_ggml(x[2 * gb:], H, I // 32))       # down
    assert np.array_equal(R.expert_convert(y, H, I, False), x)


def test_write_and_read_rows_relayout(tmp_path):
    rng = np.random.default_rng(6)
    H, I, E, L = 256, 256, 3, 2
    eb = 3 * I * (H // 32) * 18
    blobs = [_blob(rng, E * eb) for _ in range(L)]
    idx = R.write_model(tmp_path, blobs, E, 2, H, I, layout="rows")
    assert idx["version"] == 4 and idx["layout"] == "rows" and idx["dtype"] == "q4_0"
    rd = R.RelayoutReader(tmp_path)
    assert rd.layout == "rows" and rd.formats(0) == {k: "q4_0_rows" for k in ("gate", "up", "down")}
    for l in range(L):
        for e in range(E):
            g = blobs[l][e * eb:(e + 1) * eb]
            assert np.array_equal(rd.expert_blob(l, e), R.expert_convert(g, H, I, True))
            assert np.array_equal(rd.expert_ggml(l, e), g)
    rd.close()


def test_reads_the_reference_q4_k_index(tmp_path):
    # the reference relayout's own version-2 layout: Q4_K gate/up, Q6_K down (relayout.py:111-157)
    rng = np.random.default_rng(1)
    H, I, E = 512, 256, 3
    sizes = {"gate": I * (H // 256) * 144, "up": I * (H // 256) * 144, "down": H * (I // 256) * 210}
    experts = [tuple(_blob(rng, sizes[k]) for k in ("gate", "up", "down")) for _ in range(E)]
    layer = R.write_layer(tmp_path, 7, experts, {"gate": "q4_k", "up": "q4_k", "down": "q6_k"})
    index = {"magic": "NWSMOE01", "version": 2, "dtype": "q4_k", "n_layers": 1, "n_experts": E, "n_experts_used": 2,
             "embed_dim": H, "layers": {"7": layer},
             "q4_sizes": {"gate": {"out_dim": I, "in_dim": H}, "down": {"out_dim": H, "in_dim": I}}}
    (tmp_path / "index.json").write_text(json.dumps(index))
    rd = R.RelayoutReader(tmp_path)
    assert rd.version == 2 and rd.formats(7) == {"gate": "q4_k", "up": "q4_k", "down": "q6_k"}
    for e in range(E):
        ex = rd.expert(7, e)
        for k, part in zip(("gate", "up", "down"), experts[e]):
            assert np.array_equal(ex[k], part)
    with pytest.raises(ValueError):
        rd.load_into(None)                               # the HBM decode context takes q4_0 relayouts
    rd.close()


def test_rejects_foreign_directories(tmp_path):
    (tmp_path / "index.json").write_text(json.dumps({"magic": "OTHER", "layers": {}}))
    with pytest.raises(ValueError):
        R.RelayoutReader(tmp_path)


@pytest.mark.parametrize("version", [0, 1, 5, 99])
def test_rejects_unknown_versions(tmp_path, version):
    (tmp_path / "index.json").write_text(json.dumps({"magic": R.MAGIC, "version": version, "layers": {},
                                                    "n_experts": 8}))
    with pytest.raises(ValueError, match="version"):
        R.RelayoutReader(tmp_path)


@pytest.mark.gpu
def test_relayout_round_trip_through_hbm(tmp_path):
    # a model's experts written as a relayout, read back (mmap and pinned pread) into a
    # second context: the same decode, bit for bit
    import torch
    from tinygiant_b200.cache import HostTierCache
    from tinygiant_b200.engine import MoEModel
    H, I, E, k, L = 512, 256, 8, 2, 2
    rng = np.random.default_rng(2)
    m, m2 = MoEModel(H, I, E, k, L), MoEModel(H, I, E, k, L)
    m.fill_synthetic(3)
    m2.fill_synthetic(4)
    for l in range(L):
        Rl = (rng.standard_normal((E, H)) * 0.05).astype(np.float32)
        for mm in (m, m2):
            mm.set_router(l, Rl)
    blobs = [m.read_experts(l, 0, E) for l in range(L)]
    prof = {"0": {"expert_ranking": [5, 2, 7, 0, 1, 3, 4, 6], "activation_counts": [1] * 8}}
    R.write_model(tmp_path, blobs, E, k, H, I, activation_profile=prof)
    rd = R.RelayoutReader(tmp_path)
    rd.load_into(m2)
    X = torch.randn(H, device="cuda")
    a, b = X.clone(), X.clone()
    m.decode_step(a, eager=True)
    m2.decode_step(b, eager=True)
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int32), b.view(torch.int32))
    host = [rd.read_layer_pinned(l) for l in range(L)]
    assert host[0].is_pinned() and np.array_equal(host[0].numpy(), blobs[0])
    cache = HostTierCache(m2, host, cache_slots=4)
    assert cache.pin_from_profile(rd, 2) == 2          # layer 0's two hottest experts (5, 2)
    assert set(cache.pinned) == {(0, 5), (0, 2)}
    rd.close()
    m.close()
    m2.close()


@pytest.mark.gpu
def test_rows_relayout_loads_without_repack(tmp_path):
    # the host conversion gives the device repack's bytes: a "rows" relayout copied in
    # as it is reads back as the original ggml experts and decodes bit for bit alike
    import torch
    from tinygiant_b200.engine import MoEModel
    H, I, E, k, L = 512, 256, 8, 2, 2
    m, m3 = MoEModel(H, I, E, k, L), MoEModel(H, I, E, k, L)
    m.fill_synthetic(7)
    m3.fill_synthetic(8)
    rng = np.random.default_rng(9)
    for l in range(L):
        Rl = (rng.standard_normal((E, H)) * 0.05).astype(np.float32)
        m.set_router(l, Rl)
        m3.set_router(l, Rl)
    blobs = [m.read_experts(l, 0, E) for l in range(L)]
    R.write_model(tmp_path, blobs, E, k, H, I, layout="rows")
    rd = R.RelayoutReader(tmp_path)
    rd.load_into(m3)
    for l in range(L):
        assert np.array_equal(m3.read_experts(l, 0, E), blobs[l])
    X = torch.randn(H, device="cuda")
    a, b = X.clone(), X.clone()
    m.decode_step(a, eager=True)
    m3.decode_step(b, eager=True)
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int32), b.view(torch.int32))
    rd.close()
    m.close()
    m3.close()
