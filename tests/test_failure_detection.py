"""Failure detection without a GPU fault: every device wait of the library is bounded (2 s of
%globaltimer) and reports through the device error word, which fxr_check_device_error turns into
FXR_ERR_TIMEOUT. Here the end-of-frame wait of a head-split group runs on arrival slots that no rank
ever increments (a flag that nothing sets), as when a peer GPU dropped out of the group; afterwards
the same context must still run frames correctly."""
import time

import numpy as np
import pytest

import fxr
import workloads as W


@pytest.mark.gpu
def test_wait_for_a_missing_peer_times_out_and_the_context_stays_usable(cuda):
    import torch
    import oracle as O
    w = W.Workload("fd_16x16", 16, 16, 64, n_heads=4, dtype="bf16", active=0.3)
    g = fxr.head_group(2, 0, w.n_heads, w.n_tokens)
    assert g.ctas[0] > 0 and g.ctas[1] > 0
    slots = torch.zeros(16, dtype=torch.int32, device="cuda")   # this rank's arrival area
    g.arrive[0] = slots.data_ptr()
    g.arrive[1] = slots.data_ptr()
    assert fxr.check_device_error() == 0
    t0 = time.time()
    fxr.head_group_wait(g)                  # rank 1 never arrives
    with pytest.raises(fxr.FxrError) as ei:
        fxr.check_device_error()
    waited = time.time() - t0
    assert ei.value.status == fxr.FXR_ERR_TIMEOUT
    assert 1.5 < waited < 60, waited
    assert fxr.check_device_error() == 0     # reading the word cleared it

    # the context keeps working: a frame right after matches the oracle
    fr = W.make_frame(w, seed=9)
    cfg = fxr.FrameConfig(n_tokens=w.n_tokens, n_text=w.n_text, n_heads=w.n_heads, dtype="bf16",
                          rope_axes=w.rope_axes, rope_theta=w.rope_theta)
    t = {k: torch.from_numpy(fr[k]).cuda().bfloat16() for k in ("q", "k", "v", "cache_k", "cache_v", "out")}
    ws = torch.empty(fxr.workspace_size(cfg), dtype=torch.uint8, device="cuda")
    fxr.frame_forward(cfg, t["q"], t["k"], t["v"], torch.from_numpy(fr["mask"]).cuda(), None,
                      torch.from_numpy(fr["pos"]).cuda(), torch.from_numpy(fr["norm_q"]).cuda(),
                      torch.from_numpy(fr["norm_k"]).cuda(), t["cache_k"], t["cache_v"], t["out"], ws)
    assert fxr.check_device_error() == 0
    r = O.frame_forward(fr["q"], fr["k"], fr["v"], fr["mask"], None, fr["pos"], fr["norm_q"], fr["norm_k"],
                        fr["cache_k"], fr["cache_v"], fr["out"], w.n_heads, 128, w.rope_axes, w.rope_theta)
    got = t["out"].float().cpu().numpy()[r["idx"]]
    err = np.abs(got - W.round_storage(r["out"][r["idx"]], "bf16"))
    assert err.max() <= 2e-3 and err.mean() <= 2e-4, (err.max(), err.mean())
