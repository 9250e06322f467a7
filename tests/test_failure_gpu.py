"""Failure detection, tested without faulting a GPU.

1. Bounded waits: every mbarrier wait and cross-CTA flag wait in the library's
   kernels gives up after a time limit, records a code in the device error
   word and lets the kernel return. pkc_bounded_wait_check runs those wait
   helpers on a condition that never comes true (an mbarrier nobody arrives
   on, a flag nobody sets) with a 1 ms limit: the call must come back with
   PKC_ERR_KERNEL and code 108 after about that long, and the CUDA context
   must still run the encoder afterwards.
2. A failed device worker: a model opened on two device slots of one GPU
   shards a batch across two workers; PKC_FAULT_DEVICE_SLOT=1 makes slot 1's
   worker fail on the host. The call must return that failure as a status
   (PKC_ERR_INTERNAL, the message naming the slot's device), the next call
   without the fault must succeed with outputs equal bit for bit to a
   one-slot model's, and closing the model must give its device memory back.
"""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SR = 16000


def _small_model(tmp_path_factory):
    import synth
    cfg = synth.small_cfg("c2_0.6b_f16", n_layers=2, d_model=256, n_heads=4, ff_dim=1024, n_mels=80, vocab=64,
                          pred_hidden=64, joint_hidden=64)
    return synth.ensure_gguf(cfg, str(tmp_path_factory.mktemp("fail_models")))


@pytest.mark.parametrize("kind", [0, 1])
def test_bounded_wait_runs_out_and_reports(cuda, tmp_path_factory, kind):
    import pkc
    import synth
    t0 = time.perf_counter()
    st, code = pkc.bounded_wait_check(kind, 1.0)
    dt = time.perf_counter() - t0
    assert st == pkc.PKC_ERR_KERNEL, st
    assert code == 108, code
    assert dt < 5.0, dt  # 1 ms limit (+ launch), nowhere near the kernels' 2 s
    # the context is still usable: a real encode runs and is finite
    m = pkc.Model(_small_model(tmp_path_factory))
    try:
        out = m.encode_pcm_batch([synth.synth_audio(SR * 2, 3)])
    finally:
        m.close()
    assert np.isfinite(out[0]).all()


def test_failed_device_worker_returns_status(cuda, tmp_path_factory, monkeypatch):
    import torch
    import pkc
    import synth
    path = _small_model(tmp_path_factory)
    pcm = [synth.synth_audio(n, 70 + i) for i, n in enumerate([SR * 3 + 11, SR * 2, 9000, SR + 500, SR * 4])]
    one = pkc.Model(path)
    try:
        want = one.encode_pcm_batch(pcm)
    finally:
        one.close()
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    m = pkc.Model(path, devices=(0, 0))  # two workers (device slots) on one GPU
    try:
        monkeypatch.setenv("PKC_FAULT_DEVICE_SLOT", "1")
        with pytest.raises(pkc.PkcError) as e:
            m.encode_pcm_batch(pcm)
        assert e.value.status == pkc.PKC_ERR_INTERNAL and "device 0" in str(e.value) \
            and "injected" in str(e.value), str(e.value)
        monkeypatch.delenv("PKC_FAULT_DEVICE_SLOT")
        got = m.encode_pcm_batch(pcm)
    finally:
        m.close()
    for a, b in zip(got, want):
        np.testing.assert_array_equal(a, b)
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    assert free1 >= free0 - (64 << 20), (free0, free1)  # the model's memory came back
