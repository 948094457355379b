"""dm_moe_layer_noalloc (scratch in the library's fixed device array, nothing allocated)
against dm_moe_block (the context entry point) on the same layer weights and inputs.

The GPU test makes two calls in a row with different tokens: the second call starts from
whatever the first left in the scratch array, so a missed reset would show there.  Both
entry points run the same fused kernel, so the outputs agree to within NOALLOC_TOL
(rel = max|a - b| / max|b| on the MoE update y - x), and the routing (top-k ids and their
probabilities) is the same bit for bit as the context's router and the CPU oracle's on the
same input.  This file is collected last so the test also runs after every other GPU test
in the same process."""
import numpy as np
import pytest

from disk_streaming_moe_engine_b200 import DmError, Engine, RuntimeConfig, _lib, noalloc, preset, synth

NOALLOC_TOL = 1e-5


def rel(a, b):
    return float(np.abs(np.asarray(a) - np.asarray(b)).max() / max(np.abs(np.asarray(b)).max(), 1e-30))


def test_noalloc_rejects_layers_beyond_the_scratch(lib):
    """Checked on the host before any device call: H=8192, I=1024, k=16 needs more than
    the fixed 64 KiB."""
    H, I, E, k = 8192, 1024, 256, 16
    assert noalloc.scratch_bytes(H, I, k) > noalloc.SCRATCH_BYTES
    fake = 1 << 20  # never dereferenced: the size check comes first
    with pytest.raises(DmError) as ei:
        noalloc.moe_layer_noalloc(H, I, E, k, 1e-6, fake, fake, fake, fake, fake, fake + 4 * H)
    assert ei.value.code == _lib.DM_ERR_INVALID_ARG
    assert "SCRATCH_LIMIT" in ei.value.message and "65536" in ei.value.message


def _device_layer(torch, cfg, t):
    E, H, I = cfg.num_experts, cfg.hidden_size, cfg.moe_intermediate_size
    rec = [noalloc.pack_expert_record(t["gq"][e], t["gs"][e], t["gz"][e], t["uq"][e], t["us"][e], t["uz"][e],
                                      t["dq"][e], t["ds"][e], t["dz"][e], H, I) for e in range(E + 1)]
    router = np.concatenate([t["router"], t["shared_gate"][None]]).view(np.int16)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return {"router": dev(router), "post_norm": dev(t["post_norm"].view(np.int16)),
            "experts": dev(np.stack(rec[:E])), "shared": dev(rec[E])}


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["mini", "layer"])
def test_noalloc_matches_moe_block_two_calls(lib, oracle_lib, name):
    import torch

    import oracle
    cfg = preset(name)
    m = synth.synth_model(cfg, 3, layers=[0], head=False)
    t = m["layers"][0]
    H, I, E, k = cfg.hidden_size, cfg.moe_intermediate_size, cfg.num_experts, cfg.num_experts_per_tok
    assert noalloc.scratch_bytes(H, I, k) <= noalloc.SCRATCH_BYTES
    x = (np.random.default_rng(7).standard_normal((2, H)) * 3).astype(np.float32)

    om = oracle.OracleModel(m)
    with Engine(cfg, RuntimeConfig.for_context(64)) as eng:
        eng.load_model(m)
        want = eng.moe_block(x, 0)
        # the context's router on the canonically normalised input (the fused kernel's order)
        ctx_route = eng.router_forward(np.stack([oracle.rmsnorm(x[i], t["post_norm"], cfg.rms_norm_eps)
                                                 for i in range(2)]), 0)

    w = _device_layer(torch, cfg, t)
    stream = torch.cuda.current_stream().cuda_stream
    for i in range(2):
        xm = torch.from_numpy(x[i].copy()).cuda()
        y = torch.full((H,), float("nan"), dtype=torch.float32, device="cuda")
        id_d = torch.full((k,), -1, dtype=torch.int32, device="cuda")
        p_d = torch.zeros(k, dtype=torch.float32, device="cuda")
        noalloc.moe_layer_noalloc(H, I, E, k, cfg.rms_norm_eps, w["router"].data_ptr(), w["post_norm"].data_ptr(),
                                  w["experts"].data_ptr(), w["shared"].data_ptr(), xm.data_ptr(), y.data_ptr(),
                                  id_d.data_ptr(), p_d.data_ptr(), stream)
        got = y.cpu().numpy()
        assert np.isfinite(got).all()
        assert rel(got - x[i], want[i] - x[i]) < NOALLOC_TOL, (name, i)
        sel, pr = id_d.cpu().numpy(), p_d.cpu().numpy()
        _, o_ids, o_probs = oracle.moe_block(om, 0, x[i])
        np.testing.assert_array_equal(sel, o_ids)
        assert np.array_equal(pr.view(np.uint32), o_probs.view(np.uint32)), (name, i)
        np.testing.assert_array_equal(sel, ctx_route.selected_experts[i])
        assert np.array_equal(pr.view(np.uint32), ctx_route.routing_weights[i].view(np.uint32)), (name, i)
