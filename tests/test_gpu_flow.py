"""GPU parity of the device-resident SLat flow model and sampler.

One full SLat-flow forward (and a short CFG sampling run) on the CUDA path is
compared with the pinned oracle on identical seeded inputs.  Tolerance: the
north-star bound for features after one full forward, max-abs 2e-2 and
relative-L2 5e-3.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O
from pixal3d.cpp_b200.workloads import shell_coords, batched
from tests._models import random_flow_weights

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
REL_L2 = 5e-3


def check(a, e, what, max_abs=MAX_ABS, rel_l2=REL_L2):
    a = np.asarray(a, np.float64)
    e = np.asarray(e, np.float64)
    mx = float(np.abs(a - e).max())
    rl = float(np.linalg.norm(a - e) / np.linalg.norm(e))
    print(f"{what}: max_abs {mx:.3e} rel_l2 {rl:.3e}")
    assert mx <= max_abs and rl <= rel_l2, f"{what}: max_abs {mx:.3e} rel_l2 {rl:.3e}"


def two_item_coords():
    a = shell_coords(16, 5.0, 1.0)
    b = shell_coords(16, 6.0, 0.9)
    b[:, 0] = 1
    return np.ascontiguousarray(np.concatenate([a, b]))


def make(hp, seed=0, operand_dtype="f16"):
    from pixal3d.cpp_b200.flow import FlowModel, HParams
    rng = np.random.default_rng(seed)
    w = random_flow_weights(rng, hp)
    fields = {k: getattr(hp, k) for k in HParams.__dataclass_fields__ if hasattr(hp, k)}
    fh = HParams(**fields, operand_dtype=operand_dtype)
    return w, FlowModel(fh, w)


@pytest.mark.parametrize("variant", ["rope_cross", "proj", "ape"])
def test_flow_forward_reference_model(variant):
    coords = two_item_coords()
    n = coords.shape[0]
    hp = O.FlowHParams(in_channels=8, out_channels=8, model_channels=128, cond_channels=64, num_blocks=3,
                       num_heads=2, mlp_ratio=4.0,
                       proj_in_channels=7 if variant == "proj" else 0,
                       image_attn_mode="proj" if variant == "proj" else "cross",
                       pe_mode="ape" if variant == "ape" else "rope")
    w, model = make(hp, seed=1)
    rng = np.random.default_rng(2)
    x = rng.standard_normal((n, 8)).astype(np.float32)
    offs = np.array([0, 40, 77], np.int64)
    ctx = rng.standard_normal((77, 64)).astype(np.float32)
    proj = rng.standard_normal((n, 7)).astype(np.float32) if variant == "proj" else None
    ts = np.array([500.0, 250.0], np.float32)
    exp = O.slat_flow_forward(coords, x, ts, offs, ctx, proj, hp, w)
    model.prepare(torch.from_numpy(coords).cuda(), 2, (16, 16, 16), offs)
    got = model.forward(torch.from_numpy(x).cuda(), torch.from_numpy(ts).cuda(), torch.from_numpy(ctx).cuda(),
                        torch.from_numpy(proj).cuda() if proj is not None else None)
    check(got.cpu().numpy(), exp, f"flow forward [{variant}]")
    model.close()


def test_flow_forward_io_stages():
    """Benchmark config-2 layout (no reference): io resblocks + 2x down/up."""
    c0 = shell_coords(24, 8.0, 1.2)
    coords = batched(c0, 2)
    n = coords.shape[0]
    hp = O.FlowHParams(in_channels=8, out_channels=8, model_channels=128, cond_channels=64, num_blocks=2,
                       num_heads=2, io_resblocks=2, groups=32)
    w, model = make(hp, seed=3)
    rng = np.random.default_rng(4)
    x = rng.standard_normal((n, 8)).astype(np.float32)
    offs = np.array([0, 50, 100], np.int64)
    ctx = rng.standard_normal((100, 64)).astype(np.float32)
    ts = np.array([800.0, 800.0], np.float32)
    exp = O.slat_flow_forward(coords, x, ts, offs, ctx, None, hp, w)
    model.prepare(torch.from_numpy(coords).cuda(), 2, (24, 24, 24), offs)
    got = model.forward(torch.from_numpy(x).cuda(), torch.from_numpy(ts).cuda(), torch.from_numpy(ctx).cuda())
    check(got.cpu().numpy(), exp, "flow forward [io stages]")
    model.close()


@pytest.mark.parametrize("use_graph,g,gr", [(False, 3.0, 0.0), (True, 3.0, 0.0), (True, 2.35, 0.41)])
def test_flow_sample_cfg(use_graph, g, gr):
    """SLatFlowModel::sample semantics: conditional + zeros condition, CFG
    blend, optional guidance rescale, Euler steps; batch item 0 is the
    conditional image, item 1 its unconditional copy."""
    c0 = shell_coords(16, 5.5, 1.0)
    coords = batched(c0, 2)
    m = c0.shape[0]
    hp = O.FlowHParams(in_channels=8, out_channels=8, model_channels=128, cond_channels=64, num_blocks=2,
                       num_heads=2)
    w, model = make(hp, seed=5)
    rng = np.random.default_rng(6)
    noise = rng.standard_normal((m, 8)).astype(np.float32)
    ctx = rng.standard_normal((33, 64)).astype(np.float32)
    sc = O.SamplerConfig(steps=4, sigma_min=1e-5, rescale_t=3.0, guidance_strength=g, guidance_rescale=gr,
                         guidance_interval_min=0.0, guidance_interval_max=1.0)
    zctx = np.zeros_like(ctx)
    one = np.array([0, 33], np.int64)

    def ref_model(state, t, cond):
        return O.slat_flow_forward(c0, state, np.array([t], np.float32), one, ctx if cond else zctx, None, hp, w)

    exp = O.flow_euler_sample(noise, sc, ref_model, c0[:, 0].astype(np.int64), 1)
    model.prepare(torch.from_numpy(coords).cuda(), 2, (16, 16, 16), np.array([0, 33, 66]))
    xt = torch.from_numpy(noise.copy()).cuda()
    ctx2 = torch.from_numpy(np.concatenate([ctx, ctx])).cuda()
    model.sample(xt, ctx2, steps=4, guidance_strength=g, guidance_rescale=gr, rescale_t=3.0, use_graph=use_graph)
    torch.cuda.synchronize()
    check(xt.cpu().numpy(), exp, f"sample graph={use_graph} g={g} gr={gr}")
    model.close()


@pytest.mark.parametrize("use_graph", [False, True])
def test_flow_sample_concat_and_projection(use_graph):
    """The texture stage's layout (SLatFlowModel::sample with a concat
    condition and projection mode, src/slat_flow.cpp:1407-1447): each forward
    sees [state | concat]; the unconditional branch keeps the concat rows and
    zeroes the global and projected conditions."""
    c0 = shell_coords(16, 5.5, 1.0)
    coords = batched(c0, 2)
    m = c0.shape[0]
    hp = O.FlowHParams(in_channels=13, out_channels=8, model_channels=128, cond_channels=64, num_blocks=2,
                       num_heads=2, proj_in_channels=7, image_attn_mode="proj")
    w, model = make(hp, seed=7)
    rng = np.random.default_rng(8)
    noise = rng.standard_normal((m, 8)).astype(np.float32)
    concat = rng.standard_normal((m, 5)).astype(np.float32)
    proj = rng.standard_normal((m, 7)).astype(np.float32)
    ctx = rng.standard_normal((33, 64)).astype(np.float32)
    sc = O.SamplerConfig(steps=3, sigma_min=0.031, rescale_t=2.7, guidance_strength=3.0, guidance_rescale=0.0,
                         guidance_interval_min=0.0, guidance_interval_max=1.0)
    one = np.array([0, 33], np.int64)

    def ref_model(state, t, cond):
        xin = np.concatenate([state, concat], axis=1).astype(np.float32)
        return O.slat_flow_forward(c0, xin, np.array([t], np.float32), one, ctx if cond else np.zeros_like(ctx),
                                   proj if cond else np.zeros_like(proj), hp, w)

    exp = O.flow_euler_sample(noise, sc, ref_model, c0[:, 0].astype(np.int64), 1)
    model.prepare(torch.from_numpy(coords).cuda(), 2, (16, 16, 16), np.array([0, 33, 66]))
    xt = torch.from_numpy(noise.copy()).cuda()
    ctx2 = torch.from_numpy(np.concatenate([ctx, ctx])).cuda()
    model.sample(xt, ctx2, steps=3, guidance_strength=3.0, sigma_min=0.031, rescale_t=2.7, use_graph=use_graph,
                 proj=torch.from_numpy(proj).cuda(), concat=torch.from_numpy(concat).cuda())
    torch.cuda.synchronize()
    check(xt.cpu().numpy(), exp, f"sample concat+proj graph={use_graph}")
    model.close()


def test_flow_forward_bf16_operands():
    """The same forward with bf16 operands: reported, with the looser bound
    that bf16 rounding allows (the default operand type is f16)."""
    coords = two_item_coords()
    n = coords.shape[0]
    hp = O.FlowHParams(in_channels=8, out_channels=8, model_channels=128, cond_channels=64, num_blocks=3,
                       num_heads=2)
    w, model = make(hp, seed=1, operand_dtype="bf16")
    rng = np.random.default_rng(2)
    x = rng.standard_normal((n, 8)).astype(np.float32)
    offs = np.array([0, 40, 77], np.int64)
    ctx = rng.standard_normal((77, 64)).astype(np.float32)
    ts = np.array([500.0, 250.0], np.float32)
    exp = O.slat_flow_forward(coords, x, ts, offs, ctx, None, hp, w)
    model.prepare(torch.from_numpy(coords).cuda(), 2, (16, 16, 16), offs)
    got = model.forward(torch.from_numpy(x).cuda(), torch.from_numpy(ts).cuda(), torch.from_numpy(ctx).cuda())
    check(got.cpu().numpy(), exp, "flow forward [bf16 operands]", max_abs=6e-2, rel_l2=1e-2)
    model.close()


def test_flow_sample_cached_graph_and_reprepare():
    """A second sample() replays the cached step graph bit for bit.  prepare()
    on a larger coordinate set grows the workspaces; back on the smaller set
    the buffers are reused (new shape, graph re-captured); the same set again
    keeps the cached graph.  Every result matches the oracle."""
    hp = O.FlowHParams(in_channels=8, out_channels=8, model_channels=128, cond_channels=64, num_blocks=2,
                       num_heads=2)
    w, model = make(hp, seed=9)
    rng = np.random.default_rng(10)
    ctx = rng.standard_normal((21, 64)).astype(np.float32)
    ctx2 = torch.from_numpy(np.concatenate([ctx, ctx])).cuda()
    results = []
    ca, cb = shell_coords(16, 5.5, 1.0), shell_coords(20, 7.0, 1.1)
    for c0 in (ca, cb, ca, ca):
        model.prepare(torch.from_numpy(batched(c0, 2)).cuda(), 2, (20, 20, 20), np.array([0, 21, 42]))
        noise = rng.standard_normal((c0.shape[0], 8)).astype(np.float32)
        outs = []
        for _ in range(2):
            xt = torch.from_numpy(noise.copy()).cuda()
            model.sample(xt, ctx2, steps=3, guidance_strength=3.0, use_graph=True)
            outs.append(xt.cpu().numpy())
        np.testing.assert_array_equal(outs[0], outs[1])
        sc = O.SamplerConfig(steps=3, guidance_strength=3.0)
        zctx = np.zeros_like(ctx)

        def ref_model(state, t, cond):
            return O.slat_flow_forward(c0, state, np.array([t], np.float32), np.array([0, 21]), ctx if cond else zctx,
                                       None, hp, w)

        exp = O.flow_euler_sample(noise, sc, ref_model, c0[:, 0].astype(np.int64), 1)
        check(outs[0], exp, f"re-prepared sample n={c0.shape[0]}")
        results.append(outs[0])
    model.close()
