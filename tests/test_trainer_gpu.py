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
