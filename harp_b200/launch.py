"""Launching: rank files, CPU binding and the torchrun command line.

Reference: run/run.sh, run/sub.sh, run/train.sh (mpirun with a rank file from
gen_rankfile/gen_rankfile.py: 16 ranks per node, each pinned to a contiguous
block of 38 cores on its socket).  On an 8 x B200 node one rank drives one GPU;
each rank is bound to the CPU cores NVML reports as local to its GPU (the
GPU's NUMA node), split evenly between the ranks that share that node.

    python -m harp_b200.launch --nproc-per-node 8 train.py --model dit-xl-2 --synthetic --sp_size 8
    python -m harp_b200.launch rankfile hosts.txt --ranks-per-node 8     # print a rank file

The launched command runs under torchrun (--master-addr 127.0.0.1 for one
node).  Each rank calls `bind_process()` (train.py does) when HARP_BIND_CPUS=1.
"""
from __future__ import annotations

import argparse
import os
import re
import shlex
import sys
from typing import Dict, List, Optional, Sequence


def _nvml_affinity(index: int) -> Optional[List[int]]:
    try:
        import pynvml as N
    except ImportError:
        return None
    try:
        N.nvmlInit()
        try:
            h = N.nvmlDeviceGetHandleByIndex(index)
            words = (os.cpu_count() + 63) // 64
            mask = N.nvmlDeviceGetCpuAffinity(h, words)
        finally:
            N.nvmlShutdown()
    except Exception:  # noqa: BLE001 - no driver / no GPU: fall back
        return None
    cpus = []
    for w, bits in enumerate(mask):
        for b in range(64):
            if bits >> b & 1:
                cpus.append(w * 64 + b)
    return cpus or None


def cpu_sets(local_world: int, gpu_of_rank: Optional[Sequence[int]] = None,
             affinity: Optional[Dict[int, List[int]]] = None) -> List[List[int]]:
    """CPU set of each local rank: the cores local to its GPU, divided evenly
    among the local ranks whose GPUs share those cores.  Without NVML the
    machine's cores are divided evenly in rank order."""
    gpu_of_rank = list(gpu_of_rank) if gpu_of_rank is not None else list(range(local_world))
    ncpu = os.cpu_count() or 1
    if affinity is None:
        affinity = {}
        for g in set(gpu_of_rank):
            a = _nvml_affinity(g)
            if a is not None:
                affinity[g] = a
    if len(affinity) < len(set(gpu_of_rank)):
        per = max(1, ncpu // local_world)
        return [list(range(r * per, min(ncpu, (r + 1) * per))) or [r % ncpu] for r in range(local_world)]
    groups: Dict[tuple, List[int]] = {}
    for r, g in enumerate(gpu_of_rank):
        groups.setdefault(tuple(affinity[g]), []).append(r)
    out: List[List[int]] = [[] for _ in range(local_world)]
    for cpus, ranks in groups.items():
        per = max(1, len(cpus) // len(ranks))
        for i, r in enumerate(ranks):
            out[r] = list(cpus[i * per:(i + 1) * per]) or [cpus[i % len(cpus)]]
    return out


def bind_process(local_rank: Optional[int] = None, local_world: Optional[int] = None) -> Optional[List[int]]:
    """Pin this process to its share of the CPU cores local to its GPU."""
    lr = int(os.environ.get("LOCAL_RANK", "0")) if local_rank is None else local_rank
    lw = int(os.environ.get("LOCAL_WORLD_SIZE", "1")) if local_world is None else local_world
    cpus = cpu_sets(lw)[lr]
    if hasattr(os, "sched_setaffinity"):
        try:
            os.sched_setaffinity(0, set(cpus))
        except OSError:
            return None
    return cpus


def _natural_key(s: str):
    return [int(c) if c.isdigit() else c.lower() for c in re.split(r"(\d+)", s)]


def generate_rankfile(hosts: Sequence[str], ranks_per_node: int = 8, max_nodes: Optional[int] = None,
                      cores_per_node: Optional[int] = None, fmt: str = "gpu", sockets: int = 2) -> List[str]:
    """One line per rank: hosts in natural order (node2 before node10), at most
    `max_nodes` of them, `ranks_per_node` ranks per host, rank i of a host
    owning the i-th equal contiguous block of its cores.

    fmt="gpu": "rank <r>=<host> gpu=<i> cpus=<a>-<b>" (GPU i, node-wide core ids).
    fmt="mpi": the OpenMPI rankfile line "rank <r>=<host> slot=<s>:<a>-<b>",
    with socket s and core ids counted within the socket (the cores split
    evenly over `sockets`), the format the reference's launcher writes for
    mpirun (gen_rankfile/gen_rankfile.py:4-60)."""
    nodes = sorted(dict.fromkeys(h for h in hosts if h), key=_natural_key)
    if max_nodes is not None:
        nodes = nodes[:max_nodes]
    cores = cores_per_node or (os.cpu_count() or ranks_per_node)
    per = max(1, cores // ranks_per_node)
    per_socket = max(1, cores // max(1, sockets))
    lines, r = [], 0
    for host in nodes:
        for i in range(ranks_per_node):
            a, b = i * per, (i + 1) * per - 1
            if fmt == "mpi":
                lines.append(f"rank {r}={host} slot={a // per_socket}:{a % per_socket}-{b % per_socket}")
            elif fmt == "gpu":
                lines.append(f"rank {r}={host} gpu={i} cpus={a}-{b}")
            else:
                raise ValueError(f"unknown rankfile format {fmt!r} (gpu | mpi)")
            r += 1
    return lines


def torchrun_cmd(script_and_args: Sequence[str], nproc_per_node: int, nnodes: int = 1, node_rank: int = 0,
                 master_addr: str = "127.0.0.1", master_port: int = 29500) -> List[str]:
    return [sys.executable, "-m", "torch.distributed.run", f"--nnodes={nnodes}", f"--node-rank={node_rank}",
            f"--nproc-per-node={nproc_per_node}", f"--master-addr={master_addr}", f"--master-port={master_port}",
            *script_and_args]


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    if argv and argv[0] == "rankfile":
        ap = argparse.ArgumentParser(prog="harp_b200.launch rankfile")
        ap.add_argument("hostfile")
        ap.add_argument("--ranks-per-node", type=int, default=8)
        ap.add_argument("--max-nodes", type=int, default=None)
        ap.add_argument("--cores-per-node", type=int, default=None)
        ap.add_argument("--format", choices=["gpu", "mpi"], default="gpu",
                        help="gpu: GPU index and node-wide cores; mpi: OpenMPI rankfile slots (socket:cores)")
        ap.add_argument("--sockets", type=int, default=2)
        a = ap.parse_args(argv[1:])
        with open(a.hostfile) as fh:
            hosts = [ln.split()[0] for ln in fh if ln.strip()]
        print("\n".join(generate_rankfile(hosts, a.ranks_per_node, a.max_nodes, a.cores_per_node, a.format,
                                           a.sockets)))
        return 0
    ap = argparse.ArgumentParser(prog="harp_b200.launch")
    ap.add_argument("--nproc-per-node", type=int, default=8)
    ap.add_argument("--nnodes", type=int, default=1)
    ap.add_argument("--node-rank", type=int, default=0)
    ap.add_argument("--master-addr", default="127.0.0.1")
    ap.add_argument("--master-port", type=int, default=29500)
    ap.add_argument("--no-bind", action="store_true", help="do not pin ranks to GPU-local cores")
    ap.add_argument("--comm-timeout-s", type=float, default=None, help="bounded-wait limit of harp kernels")
    ap.add_argument("--dry-run", action="store_true")
    ap.add_argument("script", nargs=argparse.REMAINDER)
    a = ap.parse_args(argv)
    if not a.script:
        ap.error("missing training script")
    env = dict(os.environ)
    env.setdefault("HARP_BIND_CPUS", "0" if a.no_bind else "1")
    env.setdefault("TORCH_NCCL_ASYNC_ERROR_HANDLING", "1")
    if a.comm_timeout_s is not None:
        env["HARP_COMM_TIMEOUT_S"] = str(a.comm_timeout_s)
    cmd = torchrun_cmd(a.script, a.nproc_per_node, a.nnodes, a.node_rank, a.master_addr, a.master_port)
    if a.dry_run:
        print(" ".join(shlex.quote(c) for c in cmd))
        return 0
    os.execvpe(cmd[0], cmd, env)


if __name__ == "__main__":
    sys.exit(main())
