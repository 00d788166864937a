"""NVLink peer-memory communicator ("nvl" backend).

The B200 replacement for the reference's HMPI process group plus die-shared
memory (hmpi/ProcessGroupHMPI.cpp, gemm/ring_attention/ring_attn.cpp:1344-2410,
accumulate_sp/accumulate.cpp).  One process per GPU; torch.distributed carries
only the set-up (exchange of CUDA IPC handles); every data transfer is a
harp kernel that reads or writes peer memory over NVLink.

Synchronisation uses monotonically increasing epochs per purpose: a rank
publishes "my buffer for epoch e is ready" by storing e into its slot of every
peer's flag array (release, system scope); consumers wait until the slot is
>= e (acquire, bounded by a timeout that raises HarpDeviceError instead of
hanging).  Because epochs only grow, flags are never reset.  No kernel waits
for another kernel of the same GPU that may still be running: every wait is
for a flag that a peer GPU writes, or (own slot, or a one-rank group) that an
earlier kernel of the same stream has already written.

Inside a captured CUDA graph every flag value is step-relative: a kernel
computes it on the device as the value seen at capture plus the counter's
per-step increment times step_delta[0], which the host bumps before each
replay (begin_capture / _sd; step_value in common.cuh).

Purposes and buffers:
  KV      per-layer symmetric K|V buffers of the ring path: the QK-norm/RoPE
          kernel stores this rank's K|V chunk into every rank's buffer and
          raises KV; the attention forward waits per key tile for the flag
          of the chunk it reads, starting with its own.
  DKV     two symmetric dK|dV receive buffers (one slot per sender) used
          alternately by consecutive backward layers: the attention
          backward stores each key chunk's dK|dV into its owner's slot and
          raises DKV; the owner's reduce waits for every peer's DKV, and
          DKV_ACK tells the senders that it has summed the buffer before it
          is written again two layers later.
  GRAD / PARAM  the fused gradient reduce-scatter + AdamW + parameter push
          waits for every peer's GRAD flag; PARAM tells peers the new
          parameters have landed, which the next step waits for.
  GATH / GACK  sharded parameters (harp_b200.parallel.param_shard): each rank
          pushes its slice of a block's weights into every rank's staging
          slot s and sets GATH[s] to the slot's gather count; the GEMMs of
          that block wait for every GATH[s] (each CTA's thread 0, before its
          roles start).  A
          rank sets GACK[s] to the number of uses of slot s it has finished;
          a push into slot s first waits until every rank has finished all
          earlier uses.
  GRADB   per-bucket GRAD flags of the overlapped gradient sync: a rank sets
          its bucket-b slot from the compute stream once that bucket's
          gradients are written; the bucket's fused kernel (side stream) waits
          for every peer's slot.  Signals never wait, so ranks cannot block
          one another through the order of their side-stream kernels.
  UQKV / UO / UDO / UDQ  Ulysses exchanges, one set of symmetric buffers
          per layer (q|k|v head-sharded over the full sequence, the
          sequence-sharded attention output, dO head-sharded, dq|dk|dv
          sequence-sharded).  Each buffer is written once per step by its
          senders; the next step's writes come after every rank's gradients
          and parameters were exchanged, so no buffer needs an ack.
"""
from __future__ import annotations

import os
from typing import Dict, List, Optional

import torch
import torch.distributed as dist

from .. import _native
from ..ops import functional as Fn
from ..runtime import errors
from ..utils.observability import phase
from . import collectives as C

# flag slot layout (int32 per slot, world <= 8)
_KV, _DKV, _DKV_ACK0, _DKV_ACK1, _GRAD, _PARAM, _BARRIER = 0, 8, 16, 24, 32, 40, 48
_UQKV, _UO, _UDO, _UDQ = 56, 64, 72, 80
_GRADB = 96  # per-bucket gradient-ready slots: _GRADB + 8 * bucket + rank
_MAX_BUCKETS = 128  # flux-12b: 57 blocks, one bucket each with sharded weights
_GATH = _GRADB + 8 * _MAX_BUCKETS  # sharded parameters: slice landed in staging slot s (_GATH + 8 * s + rank)
_GACK = _GATH + 16                 # sharded parameters: uses of staging slot s completed (_GACK + 8 * s + rank)
_NFLAGS = _GACK + 16
# CTAs of one bucket's fused reduce-scatter + AdamW + push kernel: enough
# outstanding 16-byte NVLink loads to keep the links busy, few enough SMs that
# the backward it overlaps keeps most of the GPU
BUCKET_CTAS = int(os.environ.get("HARP_BUCKET_CTAS", "24"))
# HARP_ULY_PUSH=1: the Ulysses attention backward stores dK / dV straight into
# their owners' dq|dk|dv rows from its epilogue (as the ring path does) and
# only dQ goes through the remap kernel.  Off by default: not yet timed.
ULY_PUSH = os.environ.get("HARP_ULY_PUSH", "0") == "1"


def uly_dkv_push(dqkv_bases: List[int], rank: int, H: int, Dh: int, S: int) -> Dict[str, object]:
    """Arguments of the attention backward's dK/dV push for the Ulysses layout.

    The backward runs on this rank's Hn = H / W heads over the full sequence
    (W chunks of S rows per sample); key row c*S + s of local head hn belongs
    to rank c, at row b*S + s of its [B*S, 3*H*Dh] dq|dk|dv buffer, column
    H*Dh + (rank*Hn + hn)*Dh (dK) or 2*H*Dh + (rank*Hn + hn)*Dh (dV) -- the
    places the head-to-sequence remap would write.  The kernel adds
    (b*chunk + s)*ld + hn*Dh (+ vcol for dV) elements to base[c], so base[c]
    carries the column offset of this rank's heads in dK."""
    W = len(dqkv_bases)
    HD, Hn = H * Dh, H // W
    col = HD + rank * Hn * Dh  # elements
    return {"bases": [b + 2 * col for b in dqkv_bases], "chunk": S, "rank": 0, "slot": 0, "ld": 3 * HD,
            "vcol": HD}
DEFAULT_TIMEOUT_S = float(os.environ.get("HARP_COMM_TIMEOUT_S", "120"))


def available() -> bool:
    if os.environ.get("HARP_COMM", "").lower() == "torch":
        return False
    return torch.cuda.is_available() and _native.available() and hasattr(torch.ops, "harp_comm")


class SymBuffer:
    """One symmetric segment: allocated on every rank of `group` (a collective
    call: same size and order everywhere) and mapped into every peer."""

    def __init__(self, group, nbytes: int, device: torch.device):
        self.nbytes = (nbytes + 4095) // 4096 * 4096
        self.device = device
        dev = device.index
        ptr, handle = torch.ops.harp_comm.ipc_alloc(self.nbytes, dev)
        world, rank = C.world(group), C.rank(group)
        handles: List[Optional[list]] = [None] * world
        dist.all_gather_object(handles, handle.tolist(), group=group)
        self.bases: List[int] = []
        self._opened: List[int] = []
        for r in range(world):
            if r == rank:
                self.bases.append(ptr)
            else:
                p = torch.ops.harp_comm.ipc_open(torch.tensor(handles[r], dtype=torch.uint8), dev)
                self.bases.append(p)
                self._opened.append(p)
        self._own = ptr
        self.local = torch.ops.harp_comm.view(ptr, self.nbytes, torch.uint8, dev)

    def tensor(self, numel: int, dtype: torch.dtype, offset: int = 0) -> torch.Tensor:
        esz = torch.empty((), dtype=dtype).element_size()
        assert offset % esz == 0 and offset + numel * esz <= self.nbytes
        return self.local[offset:offset + numel * esz].view(dtype)

    def release(self):
        for p in self._opened:
            torch.ops.harp_comm.ipc_release(p)
        torch.ops.harp_comm.ipc_release(self._own)
        self._opened = []


class NVLinkComm:
    _instances: Dict[tuple, "NVLinkComm"] = {}

    @classmethod
    def get(cls, group, device) -> "NVLinkComm":
        key = (id(group), str(device))
        inst = cls._instances.get(key)
        if inst is None:
            inst = cls(group, torch.device(device))
            cls._instances[key] = inst
        return inst

    @classmethod
    def close_all(cls):
        for inst in list(cls._instances.values()):
            inst.close()
        cls._instances.clear()

    def __init__(self, group, device: torch.device, timeout_s: float = DEFAULT_TIMEOUT_S):
        _native.require()
        self.group, self.device = group, device
        self.world, self.rank = C.world(group), C.rank(group)
        assert self.world <= 8, "harp NVLink comm: one node, at most 8 GPUs"
        self.timeout_s = timeout_s
        self.uly_push = ULY_PUSH
        self.flags_buf = SymBuffer(group, _NFLAGS * 4, device)
        self.flags = self.flags_buf.tensor(_NFLAGS, torch.int32)
        self.flag_bases = self.flags_buf.bases
        self.epoch = {"kv": 0, "dkv": 0, "grad": 0, "barrier": 0, "uq": 0, "uo": 0, "udo": 0, "udq": 0,
                      "gath0": 0, "gath1": 0, "use0": 0, "use1": 0}
        # CUDA-graph replays of a whole step: flag values are (captured value) +
        # (increments per step of their counter) * step_delta[0]
        self.step_delta = torch.zeros(1, dtype=torch.int32, device=device)
        self._per_step: Optional[Dict[str, int]] = None
        self._uly: List[Dict[str, SymBuffer]] = []
        self._uly_idx = 0
        self._kv_idx = 0
        self._ring_bufs: List[SymBuffer] = []
        self._dkv_push: List[SymBuffer] = []
        self._dkv_idx = 0
        self._dkv_last_epoch = [0, 0]
        self._flat: Optional[Dict[str, SymBuffer]] = None
        torch.cuda.synchronize(device)
        C.all_reduce_sum_(torch.zeros(1, device=device), group)  # everyone mapped before first use

    # -- basics ---------------------------------------------------------------
    @property
    def err(self) -> torch.Tensor:
        return errors.word(self.device)

    # -- CUDA-graph capture of a step ---------------------------------------------
    def begin_capture(self, per_step: Dict[str, int]):
        """Kernels issued from now on compute their flag values on the device:
        the value at capture plus per_step[counter] * step_delta[0]."""
        self._per_step = dict(per_step)
        self.step_delta.zero_()

    def end_capture(self):
        self._per_step = None

    def _sd(self, counter: Optional[str]):
        if self._per_step is None or counter is None:
            return None, 0
        return self.step_delta, self._per_step.get(counter, 0)

    def signal(self, base: int, value: int, counter: Optional[str] = None):
        """Store `value` into slot base+rank of every rank's flag array (self included)."""
        sd, ps = self._sd(counter)
        torch.ops.harp_comm.signal([b + 4 * base for b in self.flag_bases], self.rank, value, -1, sd, ps)

    def wait_all(self, base: int, value: int, counter: Optional[str] = None):
        """Wait (on the current stream) until every rank's slot base+c >= value."""
        sd, ps = self._sd(counter)
        torch.ops.harp_comm.wait(self.flags, base, self.world, value, self.timeout_s, self.err, sd, ps)

    def barrier(self):
        self.epoch["barrier"] += 1
        e = self.epoch["barrier"]
        self.signal(_BARRIER, e, "barrier")
        self.wait_all(_BARRIER, e, "barrier")

    def begin_step(self):
        self._kv_idx = 0
        self._dkv_idx = 0
        self._uly_idx = 0

    # -- sequence-parallel ring attention: K/V pushed to every rank, dK/dV back --
    def ring_forward(self, q, k, v, B: int, S: int, H: int, Dh: int, wq=None, wk=None, freqs=None, eps: float = 1e-6,
                     do_norm: bool = False, q_ready: bool = False):
        """q, k, v: this rank's pre-norm rows [B*S, >=H*Dh] (views of one q|k|v
        tensor or separate tensors).  One kernel applies QK-norm + RoPE (when
        do_norm / freqs) and stores K, V into every rank's gathered K|V buffer
        at this rank's chunk; the attention over the full key sequence starts
        on the local chunk and takes each peer chunk as its flag arrives.
        q_ready: q is already final (no norm, no RoPE) and is used as is.
        Returns (o, q_final, rstd_q, rstd_k, saved)."""
        i = self._kv_idx
        self._kv_idx += 1
        W, r = self.world, self.rank
        HD = H * Dh
        nbytes = B * W * S * 2 * HD * 2
        while len(self._ring_bufs) <= i:
            self._ring_bufs.append(SymBuffer(self.group, nbytes, self.device))
        buf = self._ring_bufs[i]
        assert buf.nbytes >= nbytes, "ring K/V buffer shape changed between steps"
        qf = None if q_ready else torch.empty(B * S, HD, device=q.device, dtype=torch.bfloat16)
        rq = torch.empty(B * S * H, device=q.device, dtype=torch.float32) if do_norm and not q_ready else None
        rk = torch.empty(B * S * H, device=q.device, dtype=torch.float32) if do_norm else None
        self.epoch["kv"] += 1
        e = self.epoch["kv"]
        with phase("ring.dispatch_kv"):
            torch.ops.harp_comm.ring_dispatch_qkv(q, k, v, S, H, Dh, r, buf.bases, 2 * HD, qf, wq, wk, freqs,
                                                  freqs.shape[0] if freqs is not None else 1, eps, do_norm, rq, rk)
            self.signal(_KV, e, "kv")
        kv = buf.tensor(B * W * S * 2 * HD, torch.bfloat16).view(B * W * S, 2 * HD)
        qq = q if q_ready else qf
        with phase("ring.attn_fwd"):
            sd, ps = self._sd("kv")
            o, lse = Fn.attn_fwd(qq, kv[:, :HD], kv[:, HD:], B, S, W * S, H, Dh, ready=self.flags[_KV:_KV + W],
                                 chunk_len=S, start_tile=(r * S) // 128, epoch=e, timeout_s=self.timeout_s,
                                 step_delta=sd, epoch_per_step=ps)
        return o, qq, rq, rk, {"lse": lse, "kv": kv}

    def ring_backward(self, saved, q, o, do, B: int, S: int, H: int, Dh: int, out: Optional[torch.Tensor] = None,
                      out_ld: int = 0):
        """Attention backward over the gathered keys; the kernel stores the
        dK/dV rows of every chunk straight into its owner's receive buffer
        (slot = this rank), then one kernel per rank waits for every peer's
        flag and sums the slots.  Returns (dq [B*S, H*Dh], dkv): dkv is `out`
        (rows of stride out_ld holding dK at column 0, dV at H*Dh) or a new
        [B*S, 2*H*Dh] tensor."""
        W, r = self.world, self.rank
        HD = H * Dh
        slot = B * S * 2 * HD
        j = self._dkv_idx % 2
        self._dkv_idx += 1
        while len(self._dkv_push) < 2:
            self._dkv_push.append(SymBuffer(self.group, W * slot * 2, self.device))
        buf = self._dkv_push[j]
        assert buf.nbytes >= W * slot * 2, "ring dK/dV buffer shape changed between steps"
        last = self._dkv_last_epoch[j]
        if last > 0:  # every rank has summed what this buffer held two layers ago
            with phase("ring.dkv_ack_wait"):
                self.wait_all(_DKV_ACK0 if j == 0 else _DKV_ACK1, last, "dkv")
        kv = saved["kv"]
        with phase("ring.attn_bwd"):
            dq, _, _ = Fn.attn_bwd(q, kv[:, :HD], kv[:, HD:], o, do, saved["lse"], B, S, W * S, H, Dh,
                                   push={"bases": buf.bases, "chunk": S, "rank": r, "slot": slot, "ld": 2 * HD,
                                         "vcol": HD})
        self.epoch["dkv"] += 1
        e = self.epoch["dkv"]
        self.signal(_DKV, e, "dkv")
        if out is None:
            out = torch.empty(B * S, 2 * HD, device=q.device, dtype=torch.bfloat16)
            out_ld = 2 * HD
        own = buf.bases[r]
        sd, ps = self._sd("dkv")
        with phase("ring.dkv_reduce"):
            # sum of the W slots (slot c written by rank c), row by row into `out`
            torch.ops.harp_comm.reduce_scatter([own + c * slot * 2 for c in range(W)], 0, 2 * HD, out, out_ld,
                                               2 * HD, B * S, r, self.flags, _DKV, e, self.timeout_s, self.err, sd, ps)
        self._dkv_last_epoch[j] = e
        self.signal(_DKV_ACK0 if j == 0 else _DKV_ACK1, e, "dkv")
        return dq, out

    def _uly_layer(self, i: int, B: int, S: int, H: int, Dh: int) -> Dict[str, SymBuffer]:
        W = self.world
        HD, HnDh = H * Dh, (H // W) * Dh
        need = {"qkvf": 3 * B * W * S * HnDh * 2, "o": B * S * HD * 2, "dof": B * W * S * HnDh * 2,
                "dqkv": B * S * 3 * HD * 2}
        while len(self._uly) <= i:
            self._uly.append({k: SymBuffer(self.group, n, self.device) for k, n in need.items()})
        bufs = self._uly[i]
        assert all(bufs[k].nbytes >= n for k, n in need.items()), "Ulysses buffer shape changed between steps"
        return bufs

    def uly_forward(self, qkv: torch.Tensor, B: int, S: int, H: int, Dh: int, wq, wk, freqs, eps: float,
                    do_norm: bool):
        """qkv: this rank's pre-norm q|k|v rows [B*S, >=3*H*Dh].  QK-norm + RoPE
        are applied while q, k, v are written head-sharded into their owners'
        buffers; attention over the full sequence starts on the local chunk and
        takes every other chunk as its flag arrives; the output is written back
        sequence-sharded.  Returns (o [B*S, H*Dh], rstd_q, rstd_k, saved)."""
        i = self._uly_idx
        self._uly_idx += 1
        W, r = self.world, self.rank
        Hn, Sf, HD = H // W, W * S, H * Dh
        part = B * Sf * Hn * Dh
        bufs = self._uly_layer(i, B, S, H, Dh)
        rq = torch.empty(B * S * H, device=qkv.device, dtype=torch.float32) if do_norm else None
        rk = torch.empty_like(rq) if do_norm else None
        self.epoch["uq"] += 1
        e = self.epoch["uq"]
        with phase("uly.dispatch_qkv"):
            torch.ops.harp_comm.uly_dispatch_qkv(qkv, S, H, Dh, r, bufs["qkvf"].bases, part, wq, wk, freqs,
                                                 freqs.shape[0] if freqs is not None else 1, eps, do_norm, rq, rk)
            self.signal(_UQKV, e, "uq")
        qkvf = bufs["qkvf"].tensor(3 * part, torch.bfloat16).view(3, B * Sf, Hn * Dh)
        sd, ps = self._sd("uq")
        with phase("uly.attn_fwd"):
            o_f, lse = Fn.attn_fwd(qkvf[0], qkvf[1], qkvf[2], B, Sf, Sf, Hn, Dh, ready=self.flags[_UQKV:_UQKV + W],
                                   chunk_len=S, start_tile=(r * S) // 128, epoch=e, timeout_s=self.timeout_s,
                                   q_rot=(r * S) // 256, wait_q=True, step_delta=sd, epoch_per_step=ps)
        self.epoch["uo"] += 1
        eo = self.epoch["uo"]
        with phase("uly.o_remap"):
            torch.ops.harp_comm.uly_remap([o_f], 1, B, S, r, H, Dh, bufs["o"].bases, 0, HD, 0)
            self.signal(_UO, eo, "uo")
        with phase("uly.o_wait"):
            self.wait_all(_UO, eo, "uo")
        o = bufs["o"].tensor(B * S * HD, torch.bfloat16).view(B * S, HD)
        return o, rq, rk, {"i": i, "qkvf": qkvf, "o_f": o_f, "lse": lse}

    def uly_backward(self, saved, do: torch.Tensor, B: int, S: int, H: int, Dh: int) -> torch.Tensor:
        """do: dL/d(attention output) of this rank's rows [B*S, H*Dh].  Returns
        [B*S, 3*H*Dh]: dL/dq, dL/dk (after RoPE) and dL/dv of this rank's rows,
        in a buffer the caller may overwrite in place."""
        W, r = self.world, self.rank
        Hn, Sf, HD = H // W, W * S, H * Dh
        bufs = self._uly[saved["i"]]
        self.epoch["udo"] += 1
        e = self.epoch["udo"]
        with phase("uly.do_remap"):
            torch.ops.harp_comm.uly_remap([do], 0, B, S, r, H, Dh, bufs["dof"].bases, 0, 0, 0)
            self.signal(_UDO, e, "udo")
        with phase("uly.do_wait"):
            self.wait_all(_UDO, e, "udo")
        dof = bufs["dof"].tensor(B * Sf * Hn * Dh, torch.bfloat16).view(B * Sf, Hn * Dh)
        qkvf = saved["qkvf"]
        push = uly_dkv_push(bufs["dqkv"].bases, r, H, Dh, S) if self.uly_push else None
        with phase("uly.attn_bwd"):
            dq_f, dk_f, dv_f = Fn.attn_bwd(qkvf[0], qkvf[1], qkvf[2], saved["o_f"], dof, saved["lse"], B, Sf, Sf,
                                           Hn, Dh, push=push)
        self.epoch["udq"] += 1
        e2 = self.epoch["udq"]
        with phase("uly.dqkv_remap"):
            parts = [dq_f] if push is not None else [dq_f, dk_f, dv_f]
            torch.ops.harp_comm.uly_remap(parts, 1, B, S, r, H, Dh, bufs["dqkv"].bases, 0, 3 * HD, HD)
            self.signal(_UDQ, e2, "udq")
        with phase("uly.dqkv_wait"):
            self.wait_all(_UDQ, e2, "udq")
        return bufs["dqkv"].tensor(B * S * 3 * HD, torch.bfloat16).view(B * S, 3 * HD)

    # -- gradients: fused reduce-scatter + AdamW + parameter push ---------------
    def allocate_flat(self, numel: int, param_numel: Optional[int] = None):
        """Symmetric flat parameter and gradient buffers (bf16); the parameter
        buffer may be shorter (sharded parameters keep only the replicated
        ones there)."""
        pn = numel if param_numel is None else param_numel
        if self._flat is None:
            self._flat = {"param": SymBuffer(self.group, pn * 2, self.device),
                          "grad": SymBuffer(self.group, numel * 2, self.device)}
        return (self._flat["param"].tensor(pn, torch.bfloat16), self._flat["grad"].tensor(numel, torch.bfloat16))

    def wait_params(self):
        """Before touching parameters or gradients of a new step: every peer has
        pushed its updated shard (and therefore finished reading our gradients)."""
        if self.epoch["grad"] > 0:
            self.wait_all(_PARAM, self.epoch["grad"], "grad")

    def _rs_adamw_segment(self, opt, seg, slot: int, e: int, blocks: int = 0, local_out=None):
        f, n, o = seg
        cfg = opt.cfg
        sd, ps = self._sd("grad")
        torch.ops.harp_comm.rs_adamw_ag(self._flat["grad"].bases, self._flat["param"].bases, f, n,
                                        opt.master[o:o + n], opt.m[o:o + n], opt.v[o:o + n], opt.lr, cfg.beta1,
                                        cfg.beta2, cfg.eps, cfg.weight_decay, opt.step_count, cfg.grad_scale,
                                        self.rank, self.flags, slot, e, self.timeout_s, self.err, blocks, local_out,
                                        sd, ps, opt.hyper)

    def rs_adamw_ag(self, flat, opt):
        """Whole-buffer form, after backward: one signal, one fused kernel per bucket."""
        assert self._flat is not None, "flat buffers must come from allocate_flat()"
        self.epoch["grad"] += 1
        e = self.epoch["grad"]
        self.signal(_GRAD, e, "grad")
        opt.step_count += 1
        with phase("grad.rs_adamw_push"):
            for b, seg in enumerate(opt.segments):
                out = opt.local_param_out(b)
                if out is None:
                    self._rs_adamw_segment(opt, seg, _GRAD, e)
                else:
                    self._rs_adamw_local(opt, seg, _GRAD, e, out)
        self.signal(_PARAM, e, "grad")

    # -- sharded parameters: staging slots, all-gather push, acks --------------
    def param_slots(self, numel: int) -> SymBuffer:
        """Two symmetric staging slots of `numel` bf16 each (allocated once)."""
        if getattr(self, "_slots", None) is None:
            self._slots = SymBuffer(self.group, 2 * numel * 2, self.device)
            self._slot_numel = numel
        assert self._slot_numel >= numel
        return self._slots

    def slot_view(self, s: int) -> torch.Tensor:
        n = self._slot_numel
        return self._slots.tensor(2 * n, torch.bfloat16)[s * n:(s + 1) * n]

    def gather_slice(self, s: int, src: torch.Tensor, off: int):
        """Push this rank's slice `src` into offset `off` of staging slot s on
        every rank, after every rank has finished every earlier use of the
        slot; then set GATH[s] to the slot's new gather count (all on the
        current stream).  Returns that count."""
        uses = self.epoch[f"use{s}"]
        if uses > 0:
            self.wait_all(_GACK + 8 * s, uses, f"use{s}")
        n = self._slot_numel
        bases = [b + (s * n + off) * 2 for b in self._slots.bases]
        torch.ops.harp_comm.push_slice(src, bases, 0, self.rank, 32)
        self.epoch[f"gath{s}"] += 1
        self.signal(_GATH + 8 * s, self.epoch[f"gath{s}"], f"gath{s}")
        return self.epoch[f"gath{s}"]

    def gate_slot(self, s: int):
        """GEMMs launched from now on wait until every rank's GATH[s] reached
        the slot's current gather count."""
        sd, ps = self._sd(f"gath{s}")
        torch.ops.harp.set_weight_gate(self.flags, _GATH + 8 * s, self.world, self.epoch[f"gath{s}"], self.timeout_s,
                                       sd, ps)

    @staticmethod
    def clear_gate():
        torch.ops.harp.set_weight_gate(None, 0, 0, 0, 0.0)

    def ack_slot(self, s: int):
        """This rank finished one more use of staging slot s."""
        self.epoch[f"use{s}"] += 1
        self.signal(_GACK + 8 * s, self.epoch[f"use{s}"], f"use{s}")

    def _rs_adamw_local(self, opt, seg, slot: int, e: int, out: torch.Tensor, blocks: int = 0):
        self._rs_adamw_segment(opt, seg, slot, e, blocks, local_out=out)

    # overlapped form: begin_grad_sync, then rs_adamw_bucket per bucket in a
    # fixed order as gradients complete, then end_grad_sync
    def begin_grad_sync(self, opt):
        assert self._flat is not None, "flat buffers must come from allocate_flat()"
        assert len(opt.segments) <= _MAX_BUCKETS, \
            f"{len(opt.segments)} gradient buckets; the flag layout has room for {_MAX_BUCKETS}"
        self.epoch["grad"] += 1
        opt.step_count += 1

    def rs_adamw_bucket(self, flat, opt, b: int, stream: torch.cuda.Stream):
        """Bucket b's gradients are written (on the current stream): signal the
        peers from this stream, then enqueue the bucket's pull-reduce + AdamW +
        push on `stream` behind that point."""
        e = self.epoch["grad"]
        self.signal(_GRADB + 8 * b, e, "grad")
        ev = torch.cuda.Event()
        ev.record()
        stream.wait_event(ev)
        with torch.cuda.stream(stream):
            out = opt.local_param_out(b)
            if out is None:
                self._rs_adamw_segment(opt, opt.segments[b], _GRADB + 8 * b, e, BUCKET_CTAS)
            else:  # sharded parameters: the new slice stays with its owner
                self._rs_adamw_local(opt, opt.segments[b], _GRADB + 8 * b, e, out, BUCKET_CTAS)

    def end_grad_sync(self, stream: torch.cuda.Stream):
        """After the last bucket: announce the new parameters, and make the
        current stream wait for the side stream."""
        with torch.cuda.stream(stream):
            self.signal(_PARAM, self.epoch["grad"], "grad")
        torch.cuda.current_stream().wait_stream(stream)

    def close(self):
        torch.cuda.synchronize(self.device)
        uly = [b for layer in self._uly for b in layer.values()]
        slots = [self._slots] if getattr(self, "_slots", None) is not None else []
        for b in (self._ring_bufs + self._dkv_push + uly + slots +
                  list((self._flat or {}).values()) + [self.flags_buf]):
            b.release()
        self._flat, self._uly = None, []
        self._ring_bufs, self._dkv_push = [], []
        self._slots = None
