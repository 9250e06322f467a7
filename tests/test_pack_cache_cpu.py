"""CPU: the pre-pack cache (pkc_pack_cache_build, host only). The packed
weight image of a GGUF is deterministic, a second build is a cache hit that
leaves the file alone, a damaged file is rebuilt, and the cache key follows
the packing options."""
import os

import pytest


@pytest.fixture(scope="module")
def ggufs(tmp_path_factory):
    import synth
    d = str(tmp_path_factory.mktemp("m"))
    small = dict(n_layers=1, d_model=256, n_heads=4, ff_dim=256, vocab=16, pred_hidden=16, joint_hidden=16)
    return {
        "f16": synth.ensure_gguf(synth.small_cfg("c2_0.6b_f16", **small), d),
        "q8_0": synth.ensure_gguf(synth.small_cfg("c3_0.6b_q8", n_mels=80, **small), d),
    }


@pytest.mark.parametrize("kind", ["f16", "q8_0"])
def test_pack_cache_build_hit_and_repair(ggufs, tmp_path, kind):
    import pkc
    a, b = tmp_path / "a", tmp_path / "b"
    a.mkdir()
    b.mkdir()
    p = pkc.pack_cache_build(ggufs[kind], str(a))
    assert os.path.dirname(p) == str(a) and os.path.getsize(p) > 4096
    t0 = os.stat(p).st_mtime_ns
    assert pkc.pack_cache_build(ggufs[kind], str(a)) == p
    assert os.stat(p).st_mtime_ns == t0          # a hit: not rewritten
    q = pkc.pack_cache_build(ggufs[kind], str(b))
    good = open(q, "rb").read()
    assert open(p, "rb").read() == good          # the packed image is deterministic
    with open(p, "r+b") as f:                    # truncated: rebuilt
        f.truncate(len(good) // 2)
    assert pkc.pack_cache_build(ggufs[kind], str(a)) == p
    assert open(p, "rb").read() == good
    with open(p, "r+b") as f:                    # foreign header: rebuilt
        f.write(b"NOTAPACK")
    assert pkc.pack_cache_build(ggufs[kind], str(a)) == p
    assert open(p, "rb").read() == good


def test_pack_cache_key_follows_model_and_options(ggufs, tmp_path, monkeypatch):
    import pkc
    p16 = pkc.pack_cache_build(ggufs["f16"], str(tmp_path))
    p8 = pkc.pack_cache_build(ggufs["q8_0"], str(tmp_path))
    assert p16 != p8
    monkeypatch.setenv("PKC_DEQUANT_AT_LOAD", "1")   # q8_0 dequantised on the host: another image
    p8d = pkc.pack_cache_build(ggufs["q8_0"], str(tmp_path))
    assert p8d != p8
    assert os.path.getsize(p8d) > os.path.getsize(p8)


def test_pack_cache_build_errors(tmp_path):
    import pkc
    with pytest.raises(pkc.PkcError) as e:
        pkc.pack_cache_build(str(tmp_path / "missing.gguf"), str(tmp_path))
    assert e.value.status == 2   # PKC_ERR_IO
