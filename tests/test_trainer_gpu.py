"""The trainer's CUDA-graph mode: the captured step replays exactly the eager
step (same kernels, same inputs, AdamW hyper-parameters read from the device)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _model():
    from harp_b200.models.dit import DiT, PRESETS

    m = DiT(PRESETS["small"])
    m.initialize_weights(0)
    return m.to(torch.bfloat16)


def _batches(n, cfg, B=2, L=16, T=8):
    g = torch.Generator().manual_seed(7)
    out = []
    for _ in range(n):
        out.append({"latent": torch.randn(B, cfg.in_channels, L, L, generator=g).to(torch.bfloat16).pin_memory(),
                    "noise": torch.randn(B, cfg.in_channels, L, L, generator=g).to(torch.bfloat16).pin_memory(),
                    "text": torch.randn(B, T, cfg.text_dim, generator=g).to(torch.bfloat16).pin_memory(),
                    "sigmas": torch.rand(B, generator=g).pin_memory()})
    return out


def test_cuda_graph_step_matches_eager():
    import harp_b200
    from harp_b200.trainer import ParallelState, TrainConfig, Trainer

    assert harp_b200.load_native(build_if_needed=True)
    dev = torch.device("cuda", 0)
    results = {}
    for graph in (False, True):
        model = _model().to(dev)
        tr = Trainer(model, ParallelState.build(1), TrainConfig(lr=1e-3, cuda_graph=graph, graph_warmup=2), dev)
        batches = _batches(6, model.cfg)
        losses = [tr.step(b) for b in batches]
        tr.check_errors()
        results[graph] = (losses, tr.flat.flat.clone(), tr.opt.step_count)
        if graph:
            assert tr._graph is not None and tr._graph_launches > 0
    (le, fe, se), (lg, fg, sg) = results[False], results[True]
    assert se == sg == 6
    assert le == lg, (le, lg)
    assert torch.equal(fe, fg)


def test_offloaded_optimizer_and_activations_match_device_resident():
    """fp32 master/m/v in pinned host memory (read by the AdamW kernel over the
    host link) and activations parked in host memory between forward and
    backward give the same steps as everything on the device."""
    import harp_b200
    from harp_b200.trainer import ParallelState, TrainConfig, Trainer

    assert harp_b200.load_native(build_if_needed=True)
    dev = torch.device("cuda", 0)
    results = {}
    for off in (False, True):
        model = _model().to(dev)
        cfg = TrainConfig(lr=1e-3, offload_optimizer=off, offload_activations=off)
        tr = Trainer(model, ParallelState.build(1), cfg, dev)
        if off:
            # the optimizer state really lives in host memory (mapped for the kernels)
            from harp_b200.runtime import alloc

            assert alloc.stats("host")["in_use"] >= 3 * tr.opt.master.numel() * 4
        losses = [tr.step(b) for b in _batches(3, model.cfg)]
        tr.check_errors()
        results[off] = (losses, tr.flat.flat.clone(), tr.opt.master.clone())
    (l0, f0, m0), (l1, f1, m1) = results[False], results[True]
    assert l0 == l1, (l0, l1)
    assert torch.equal(f0, f1) and torch.equal(m0.cpu(), m1.cpu())
