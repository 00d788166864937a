"""Kernel microbenchmarks on the DiT-XL/2 training shapes.

    python -m harp_b200.ops.microbench [case ...] [--iters N] [--small] [--no-ref]

Cases: gemm_qkv gemm_proj gemm_w13 gemm_w2 gemm_dw13 gemm_dx2 attn_fwd attn_bwd
attn_fwd_d128 attn_bwd_d128 rmsnorm_fwd rmsnorm_bwd qknorm_fwd qknorm_bwd swiglu_fwd
adamw (default: all).  Each case runs the harp kernel and, unless --no-ref,
the library path of the same op (cuBLAS through torch.matmul, SDPA for
attention).  Timing: CUDA events on the launching stream around each launch,
after 3 warm-up launches, with a 512 MiB write between timed launches so every
launch starts from a cold L2 (126 MB).  Achieved TFLOP/s and GB/s are divided
by MEASURED_PEAKS.json (copy bandwidth; cuBLAS bf16 burst) when present.
--small shrinks the shapes for ncu captures (inputs still larger than L2 for
the memory-bound cases).  One JSON line per case.
"""
from __future__ import annotations

import argparse
import json
import os
from typing import Callable, Dict

import torch

from . import functional as Fn

B, S, D, H, Dh, F_ = 4, 4352, 1152, 16, 72, 4608


def _peaks() -> Dict[str, float]:
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                     "MEASURED_PEAKS.json")
    try:
        with open(p) as fh:
            d = json.load(fh)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "src": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


class Timer:
    def __init__(self):
        self.flush = torch.empty(512 << 20, dtype=torch.uint8, device="cuda")

    def __call__(self, fn: Callable[[], None], iters: int, warmup: int = 3) -> float:
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        tot = 0.0
        for _ in range(iters):
            self.flush.fill_(1)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            tot += a.elapsed_time(b)
        return tot / iters


def _r(*shape, scale=1.0):
    return (torch.randn(*shape, device="cuda") * scale).to(torch.bfloat16)


def gemm_case(M, N, K, a_mn=False, b_mn=False):
    def make():
        a = _r(K, M) if a_mn else _r(M, K)
        b = _r(K, N) if b_mn else _r(N, K)
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        harp = lambda: Fn.gemm(a, b, a_mn=a_mn, b_mn=b_mn, out=out)  # noqa: E731
        am = a.t() if a_mn else a
        bm = b if b_mn else b.t()
        ref = lambda: torch.matmul(am, bm, out=out)  # noqa: E731
        return harp, ref, {"flops": 2.0 * M * N * K, "shape": [M, N, K], "a_mn": a_mn, "b_mn": b_mn}
    return make


def attn_case(fwd: bool, dh: int, heads: int):
    def make():
        T = B * S
        q, k, v = _r(T, heads * dh), _r(T, heads * dh), _r(T, heads * dh)
        o, lse = Fn.attn_fwd(q, k, v, B, S, S, heads, dh)
        do = _r(T, heads * dh)
        qh, kh, vh = (t.view(B, S, heads, dh).transpose(1, 2) for t in (q, k, v))
        flops = 4.0 * B * heads * S * S * dh * (1.0 if fwd else 2.5)
        if fwd:
            harp = lambda: Fn.attn_fwd(q, k, v, B, S, S, heads, dh, out=o)  # noqa: E731
            ref = lambda: torch.nn.functional.scaled_dot_product_attention(qh, kh, vh)  # noqa: E731
        else:
            dq = torch.empty_like(q)
            dk = torch.empty_like(k)
            dv = torch.empty_like(v)
            harp = lambda: Fn.attn_bwd(q, k, v, o, do, lse, B, S, S, heads, dh, dq_out=dq, dk_out=dk,  # noqa: E731
                                       dv_out=dv)
            qr, kr, vr = (t.detach().clone().requires_grad_(True) for t in (qh, kh, vh))
            orf = torch.nn.functional.scaled_dot_product_attention(qr, kr, vr)
            dor = do.view(B, S, heads, dh).transpose(1, 2)
            ref = lambda: torch.autograd.grad(orf, (qr, kr, vr), dor, retain_graph=True)  # noqa: E731
        return harp, ref, {"flops": flops, "shape": [B, S, heads, dh]}
    return make


def rmsnorm_case(bwd: bool):
    def make():
        R = B * S
        x = _r(R, D)
        sc, sh = _r(B, D, scale=0.1), _r(B, D, scale=0.1)
        y, rstd = Fn.rmsnorm_mod_fwd(x, None, sc, sh, S, 1e-6)
        dy = _r(R, D)
        if not bwd:
            harp = lambda: Fn.rmsnorm_mod_fwd(x, None, sc, sh, S, 1e-6, out=y)  # noqa: E731
            nbytes = 2 * R * D * 2
            ref = lambda: torch.nn.functional.rms_norm(x, (D,), None, 1e-6)  # noqa: E731
        else:
            harp = lambda: Fn.rmsnorm_mod_bwd(x, rstd, dy, None, sc, S, dres=dy, want_mod=True)  # noqa: E731
            nbytes = 4 * R * D * 2
            ref = None
        return harp, ref, {"bytes": nbytes, "shape": [R, D]}
    return make


def gate_case():
    def make():
        R = B * S
        dy, a, g = _r(R, D), _r(R, D), _r(B, D, scale=0.1)
        harp = lambda: Fn.gate_bwd(dy, a, g, S, want_bias=True)  # noqa: E731
        return harp, None, {"bytes": 3 * R * D * 2, "shape": [R, D]}
    return make


def qknorm_case(bwd: bool):
    def make():
        from ..models.dit import joint_positions, rope_freqs

        R = B * S
        qkv = _r(R, 3 * D)
        wq = torch.ones(Dh, device="cuda", dtype=torch.bfloat16)
        wk = torch.ones_like(wq)
        freqs = rope_freqs(joint_positions(64, 64, 256), (8, 32, 32), 10000.0).cuda()
        q, k, rq, rk = Fn.qknorm_rope_fwd(qkv, H, Dh, wq, wk, freqs, 1e-6)
        if not bwd:
            harp = lambda: Fn.qknorm_rope_fwd(qkv, H, Dh, wq, wk, freqs, 1e-6)  # noqa: E731
            nbytes = 4 * R * D * 2
        else:
            dq, dk = _r(R, D), _r(R, D)
            dqkv = torch.empty_like(qkv)
            harp = lambda: Fn.qknorm_rope_bwd(dq, dk, qkv, rq, rk, H, Dh, wq, wk, freqs, True, dqkv)  # noqa: E731
            nbytes = 6 * R * D * 2
        return harp, None, {"bytes": nbytes, "shape": [R, H, Dh]}
    return make


def swiglu_case():
    def make():
        R = B * S
        gu = _r(R, 2 * F_)
        harp = lambda: Fn.swiglu_fwd(gu, F_)  # noqa: E731
        g, u = gu[:, :F_], gu[:, F_:]
        ref = lambda: torch.nn.functional.silu(g) * u  # noqa: E731
        return harp, ref, {"bytes": 3 * R * F_ * 2, "shape": [R, F_]}
    return make


def adamw_case(n):
    def make():
        master = torch.randn(n, device="cuda")
        m = torch.zeros_like(master)
        v = torch.zeros_like(master)
        g = _r(n, scale=1e-3)
        p = master.to(torch.bfloat16)
        harp = lambda: Fn.adamw_flat(master, m, v, g, p, 1e-4, 0.9, 0.999, 1e-8, 0.0, 1)  # noqa: E731
        # master, m, v read+write (fp32), grad read (bf16), param write (bf16)
        return harp, None, {"bytes": n * (3 * 4 * 2 + 2 + 2), "shape": [n]}
    return make


def build_cases(gemm_rows: int, adamw_n: int) -> Dict[str, Callable]:
    return {
        "gemm_qkv": gemm_case(gemm_rows, 3 * D, D),
        "gemm_proj": gemm_case(gemm_rows, D, D),
        "gemm_w13": gemm_case(gemm_rows, 2 * F_, D),
        "gemm_w2": gemm_case(gemm_rows, D, F_),
        "gemm_dw13": gemm_case(2 * F_, D, gemm_rows, a_mn=True, b_mn=True),
        "gemm_dx2": gemm_case(gemm_rows, F_, D, b_mn=True),
        "attn_fwd": attn_case(True, Dh, H),
        "attn_bwd": attn_case(False, Dh, H),
        "attn_fwd_d128": attn_case(True, 128, 24),
        "attn_bwd_d128": attn_case(False, 128, 24),
        "rmsnorm_fwd": rmsnorm_case(False),
        "rmsnorm_bwd": rmsnorm_case(True),
        "gate_bwd": gate_case(),
        "qknorm_fwd": qknorm_case(False),
        "qknorm_bwd": qknorm_case(True),
        "swiglu_fwd": swiglu_case(),
        "adamw": adamw_case(adamw_n),
    }


def fwd_timeline(fn) -> Dict[str, float]:
    """Median phase durations (SM cycles) of CTA 0 of one forward launch, from
    the probe slots the forward kernels record per key step: 0/1 the MMA warp
    sees P of query tile 0/1, 4/7 the softmax warps of tile 0/1 see S, 10/11
    their TMEM loads landed, 12/13 exponentials done, 6/9 P handed over."""
    torch.cuda.synchronize()
    torch.ops.harp.attn_bwd_probe()  # clears the slots
    fn()
    torch.cuda.synchronize()
    t = torch.ops.harp.attn_bwd_probe().double()
    steps = int((t[:, 4] > 0).sum().item())
    d = t[2:max(3, steps - 1)]  # steady state: skip the first two and the last key steps

    def med(a, b):
        return round((d[:, b] - d[:, a]).median().item(), 1)

    return {"key_steps": steps, "period": round((t[3:steps, 4] - t[2:steps - 1, 4]).median().item(), 1),
            "s_seen_to_loads": med(4, 10), "loads_to_exp_done": med(10, 12), "exp_done_to_p_ready": med(12, 6),
            "p_ready_to_mma_sees_p": med(6, 0), "mma_sees_p_to_next_s_seen": round(
                (t[3:steps, 4] - t[2:steps - 1, 0]).median().item(), 1)}


def bwd_timeline(fn) -> Dict[str, float]:
    """Median per-query-tile phase durations (SM cycles) of CTA 0 of one
    backward launch (128-query pipelined schedule).  Probe slots per tile i:
    10 the TMA warp issues the Q/dO loads, 0 the MMA warp has issued S/dP,
    4 the dS warps see S/dP, 11 their TMEM loads landed, 12 P/dS computed,
    13 the previous tile's products released P/dS, 5 P/dS stored, 1 the MMA
    warp sees P/dS, 3 dV/dK/dQ issued, 6 the dQ warps see dQ, 7 dQ staged,
    9 its reduce-add has read the staging buffer."""
    torch.cuda.synchronize()
    torch.ops.harp.attn_bwd_probe()
    fn()
    torch.cuda.synchronize()
    t = torch.ops.harp.attn_bwd_probe().double()
    tiles = int((t[:, 4] > 0).sum().item())
    lo, hi = 2, max(3, tiles - 1)
    d = t[lo:hi]

    def med(a, b, shift=0):
        return round((t[lo + shift:hi + shift, b] - d[:, a]).median().item(), 1)

    out = {"tiles": tiles, "period": round((t[lo + 1:hi + 1, 4] - d[:, 4]).median().item(), 1)}
    for name, a, b in (("load_issue_to_s_issued", 10, 0), ("s_issued_to_ds_sees_s", 0, 4),
                       ("ds_sees_s_to_loaded", 4, 11), ("loaded_to_computed", 11, 12),
                       ("computed_to_prev_free", 12, 13), ("prev_free_to_stored", 13, 5),
                       ("stored_to_mma_sees_p", 5, 1), ("mma_sees_p_to_issued", 1, 3),
                       ("issued_to_dq_seen", 3, 6), ("dq_seen_to_staged", 6, 7), ("staged_to_reduced", 7, 9)):
        out[name] = med(a, b)
    out["ds_compute_cycles"] = round(d[:, 14].median().item(), 1)
    return out


def main(argv=None):
    global B, S
    ap = argparse.ArgumentParser()
    ap.add_argument("cases", nargs="*")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--small", action="store_true", help="batch 1, 2048 tokens (ncu captures)")
    ap.add_argument("--no-ref", action="store_true")
    ap.add_argument("--gemm-single", action="store_true",
                    help="also time GEMM cases with CTA-pair tiles switched off (harp1)")
    ap.add_argument("--timeline", action="store_true",
                    help="attention cases: also print the per-key-step (forward) or per-query-tile "
                         "(backward) phase timeline of CTA 0 (SM cycles)")
    args = ap.parse_args(argv)
    if args.timeline:
        os.environ["HARP_ATTN_PROBE"] = "1"  # read by the library at its first attention launch
    from .. import _native

    _native.require()
    if args.small:
        B, S = 1, 2048
    cases = build_cases(4 * B * S if args.small else B * S, 64_000_000 if args.small else 675_000_000)
    peaks = _peaks()
    timer = Timer()
    for name in args.cases or list(cases):
        harp, ref, info = cases[name]()
        rec = {"case": name, **info}
        single = args.gemm_single and name.startswith("gemm")
        for tag, fn in (("harp", harp), ("harp1", harp if single else None),
                        ("ref", None if args.no_ref else ref)):
            if fn is None:
                continue
            prev = torch.ops.harp.gemm_pair_mode(0) if tag == "harp1" else None
            try:
                ms = timer(fn, args.iters)
            finally:
                if prev is not None:
                    torch.ops.harp.gemm_pair_mode(prev)
            rec[f"{tag}_ms"] = round(ms, 4)
            if "flops" in info:
                tf = info["flops"] / ms / 1e9
                rec[f"{tag}_tflops"] = round(tf, 1)
                rec[f"{tag}_frac_of_{peaks['src']}_bf16"] = round(tf / peaks["bf16_tflops"], 3)
            else:
                gbs = info["bytes"] / ms / 1e6
                rec[f"{tag}_gbs"] = round(gbs, 1)
                rec[f"{tag}_frac_of_{peaks['src']}_hbm"] = round(gbs / peaks["hbm_gbs"], 3)
        if args.timeline and name.startswith("attn_fwd"):
            rec["timeline_cycles"] = fwd_timeline(harp)
        elif args.timeline and name.startswith("attn_bwd"):
            rec["timeline_cycles"] = bwd_timeline(harp)
        print(json.dumps(rec), flush=True)
        del harp, ref
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
