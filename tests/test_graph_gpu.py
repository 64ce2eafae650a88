"""Projection launches captured into a CUDA graph (the graph runner of the
DiT forward replays them every sampler step): a launch with the fused LoRA
prologue, whose tiles wait on ready flags set by other CTA pairs, replays
with the bits of the same eager launch, input after input (a replay that saw
the flags of the previous one would read a stale rank-space intermediate);
the state version moves with every strength or binding change."""
import numpy as np
import pytest
import torch

from mingproj.dit import _device_affine

pytestmark = pytest.mark.gpu

RANKS = (4, 8, 8, 16, 16, 32, 32, 64)
H = 3840


def _bits(t):
    return t.view(torch.int16)


def test_fused_prologue_replays_bit_identical(ctx):
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(7)
    ws = []
    for _ in range(3):
        c, sc, bi = _device_affine(gen, H, H, 8, dev)
        ws.append(ctx.upload(H, H, 8, c, sc, bi))
    for w in ws:
        for slot, r in enumerate(RANKS):
            a = (torch.randn((r, H), device=dev, generator=gen) / r ** 0.5).to(torch.bfloat16)
            b = (torch.randn((H, r), device=dev, generator=gen) * 0.01).to(torch.bfloat16)
            w.bind(slot, a, b)
    v0 = ctx.state_version()
    strengths = np.random.default_rng(3).uniform(-1.0, 1.5, size=8)
    for i, s in enumerate(strengths):
        ctx.set_strength(i, float(s))
    assert ctx.state_version() > v0
    x = torch.randn((4352, H), device=dev, generator=gen).to(torch.bfloat16)
    try:
        # a row count whose launch takes the fused prologue (one kernel, with
        # its rank-space pre-GEMM inside)
        m = None
        for rows in (4352, 4096, 3584, 3072, 2560, 2048):
            ctx.reset_engagement()
            ctx.linear_shared(ws, x[:rows])
            torch.cuda.synchronize(dev)
            e = ctx.engagement()
            if e["kernels"] == 1 and e["lora_down"] == 1:
                m = rows
                break
        assert m is not None, "no row count took the fused prologue"
        xs = x[:m].clone()
        outs = [torch.empty((m, H), dtype=torch.bfloat16, device=dev) for _ in ws]
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            ctx.linear_shared(ws, xs, outs=outs)
        torch.cuda.current_stream(dev).wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            ctx.linear_shared(ws, xs, outs=outs)
        for trial in range(3):
            xs.copy_(torch.randn((m, H), device=dev, generator=gen).to(torch.bfloat16))
            g.replay()
            ref = ctx.linear_shared(ws, xs)
            torch.cuda.synchronize(dev)
            for o, r in zip(outs, ref):
                assert torch.equal(_bits(o), _bits(r)), f"replay {trial} differs"
        del g
        ctx.sync_check()
    finally:
        for i in range(8):
            ctx.set_strength(i, 1.0)
        for w in ws:
            w.free()


def test_side_stream_lora_chain_replays_bit_identical(ctx):
    """A split-K projection over few rows with live slots forks a side stream
    (rank-space pre-GEMM, its reduce and the LoRA split) and joins it before
    the final reduce: captured into a CUDA graph, the fork and join are graph
    edges, and every replay gives the bits of the same eager call."""
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(11)
    m = 256
    c, sc, bi = _device_affine(gen, H, H, 8, dev)
    w = ctx.upload(H, H, 8, c, sc, bi)
    for slot in range(8):
        a = (torch.randn((32, H), device=dev, generator=gen) / 32 ** 0.5).to(torch.bfloat16)
        b = (torch.randn((H, 32), device=dev, generator=gen) * 0.01).to(torch.bfloat16)
        w.bind(slot, a, b)
    strengths = np.random.default_rng(5).uniform(-1.0, 1.5, size=8)
    for i, s in enumerate(strengths):
        ctx.set_strength(i, float(s))
    try:
        xs = torch.randn((m, H), device=dev, generator=gen).to(torch.bfloat16)
        ctx.reset_engagement()
        ctx.linear(w, xs)
        torch.cuda.synchronize(dev)
        # pre-GEMM, its reduce, LoRA split, base splits, final reduce (the
        # sequential form is four launches: no LoRA split of its own)
        assert ctx.engagement()["kernels"] == 5, "the side-stream chain did not run"
        out = torch.empty((m, H), dtype=torch.bfloat16, device=dev)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            ctx.linear(w, xs, out)
        torch.cuda.current_stream(dev).wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            ctx.linear(w, xs, out)
        for trial in range(3):
            xs.copy_(torch.randn((m, H), device=dev, generator=gen).to(torch.bfloat16))
            g.replay()
            ref = ctx.linear(w, xs)
            torch.cuda.synchronize(dev)
            assert torch.equal(_bits(out), _bits(ref)), f"replay {trial} differs"
        del g
        ctx.sync_check()
    finally:
        for i in range(8):
            ctx.set_strength(i, 1.0)
        w.free()


def test_side_stream_first_use_inside_a_capture():
    """The side stream, its events and the partial-sum buffers are created by
    the first split-K call with live slots; when that first call is made
    inside a CUDA-graph capture, the capture holds it and replays the eager
    bits."""
    from mingproj.proj import Context
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(13)
    c2 = Context(0)
    m = 256
    try:
        cc, sc, bi = _device_affine(gen, H, H, 8, dev)
        w = c2.upload(H, H, 8, cc, sc, bi)
        for slot in range(8):
            a = (torch.randn((32, H), device=dev, generator=gen) / 32 ** 0.5).to(torch.bfloat16)
            b = (torch.randn((H, 32), device=dev, generator=gen) * 0.01).to(torch.bfloat16)
            w.bind(slot, a, b)
            c2.set_strength(slot, 0.25 * (slot - 3))
        xs = torch.randn((m, H), device=dev, generator=gen).to(torch.bfloat16)
        out = torch.empty((m, H), dtype=torch.bfloat16, device=dev)
        torch.cuda.synchronize(dev)
        c2.reset_engagement()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            c2.linear(w, xs, out)
        assert c2.engagement()["kernels"] == 5, "the side-stream chain was not captured"
        g.replay()
        ref = c2.linear(w, xs)
        torch.cuda.synchronize(dev)
        assert torch.equal(_bits(out), _bits(ref))
        del g
        c2.sync_check()
        w.free()
    finally:
        c2.close()
