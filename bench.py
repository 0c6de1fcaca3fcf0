"""Benchmark of the E2Former-V2 energy + forces evaluation on B200 (the path's headline metric).

Default workload (``--workload model``): the full-size random-init E2Former-V2 backbone (4 layers,
node irreps 256x0e+256x1e+256x2e, 128 heads, 8 scalar dims, head irreps 2x0e+2x1e+2x2e, 256 RBF,
cutoff 6 A, at most 32 neighbours) on a ~1e5-atom periodic system (a seeded 8,000-atom H/C/N/O/S
blob in rigid water, 100 A cube).  One step = one energy + forces evaluation as the MD / ASE
interfaces call it: CUDA PBC images, radius graph and CSR, Wigner matrices, the backbone, the
energy head and forces = -dE/dpos by autograd.  fp32 throughout (3xTF32 tensor-core GEMMs).
Metric: atom-steps/s = atoms x steps / device seconds.  ``--workload layer`` is the isolated
attention-layer microbenchmark (one layer forward + backward on a uniform box).

* ``value``: positions resident in HBM, CUDA events around exactly K steps, barrier + synchronize
  on both sides, max over ranks.  All inputs are larger than L2.
* ``e2e``: the same step through the public API (``E2FormerPotential.forward``) from pinned HOST
  buffers each step: H2D of positions and atomic numbers, D2H of energy and forces.
* ``roofline``: the dominant attention kernel entry point of this package, timed with CUDA events on
  its launch stream inside the timed region, against its compulsory (algorithmic) bytes.
* ``cpu_baseline``: the CPU oracle (the reference algorithm restated) on a bounded sample.

Multi-GPU: ``--gpus N`` under torchrun splits the one ~1e5-atom system into N slabs (spatial domain
decomposition with a per-layer halo exchange of boundary-atom features over NCCL; ``scaling:
strong``); ``--replicas`` (and the layer workload) runs one independent system per rank (``weak``).
``--impl reference`` times the CPU restatement of the reference path (the reference itself is pure
Python and is not installed on the GPU box).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch

# growable allocator segments (set before the first device allocation): graph-sized tensors change size
# every MD step, which fragments fixed segments near the device's capacity
os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

C_CH, HEADS, DHEAD, NB, CUTOFF = 256, 128, 8, 256, 6.0
HEAD_IRREPS = "2x0e+2x1e+2x2e"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="model", choices=["model", "layer", "molecules", "span", "gemm", "md"])
    ap.add_argument("--molecules", type=int, default=4096, help="molecules workload: batch size")
    ap.add_argument("--atoms", type=int, default=100_000, help="layer workload: atoms")
    ap.add_argument("--k", type=int, default=32)
    ap.add_argument("--edge-chunk", type=int, default=None,
                    help="layer workload: run the edge side in checkpointed row blocks of about this many edges "
                         "(the radial basis is then formed inside its GEMM, not a leaf)")
    ap.add_argument("--cpu-atoms", type=int, default=None,
                    help="CPU baseline sample size (default 500 for the model, 1500 for the layer)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--projections", default="fp32", choices=["fp32", "tf32"],
                    help="model workload: fp32-accurate 3xTF32 projections (parity, the headline) or the "
                         "single-pass TF32 mode (the reference's use_tf32)")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--replicas", action="store_true",
                    help="model workload with N > 1: independent systems per rank instead of one system "
                         "split into slabs (domain decomposition)")
    return ap.parse_args()


# ------------------------------------------------------------------------------------------------
def dist_init(args):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import torch.distributed as dist
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        dist.init_process_group(backend=backend)
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, ws, dev):
    if ws == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def config_dict(args, E=None, N2=None, extra=None):
    d = {"workload": f"E2AttentionArbOrder_sparse forward+backward, periodic uniform box {args.atoms} atoms, "
                     f"~{args.k} neighbours within {CUTOFF} A",
         "atoms_per_rank": args.atoms, "k_avg": args.k, "irreps": f"{C_CH}x0e+{C_CH}x1e+{C_CH}x2e",
         "heads": HEADS, "attn_scalar_head": DHEAD, "irreps_head": HEAD_IRREPS, "rbf": NB, "cutoff": CUTOFF,
         "l2": "inputs larger than L2 (value rows alone are GBs)", "parallelism": f"replicas x{args.gpus}"}
    if getattr(args, "edge_chunk", None):
        d["edge_chunk"] = args.edge_chunk
    if E is not None:
        d["edges_per_rank"] = E
        d["expanded_nodes_per_rank"] = N2
    if extra:
        d.update(extra)
    return d


# ------------------------------------------------------------------------------------------------
def make_layer(dev, seed=0):
    from ubio_molfm_b200.attention import E2AttentionArbOrder_sparse
    from ubio_molfm_b200.synthetic import seeded_params_

    layer = E2AttentionArbOrder_sparse(f"{C_CH}x0e+{C_CH}x1e+{C_CH}x2e", NB, num_attn_heads=HEADS,
                                       attn_scalar_head=DHEAD, irreps_head=HEAD_IRREPS, alpha_drop=0.0,
                                       tp_type="QK_alpha+triton", attn_type="so2-first-order")
    seeded_params_(layer, seed)
    return layer.to(dev).eval()


def build_inputs(pos, Z, cell, dev, layer, materialize_rbf=True):
    """Graph + per-node geometry for one periodic system (all on ``dev``)."""
    from ubio_molfm_b200.graph import expand_pbc, radius_graph
    from ubio_molfm_b200.nn import GaussianSmearing
    from ubio_molfm_b200.wigner import node_wigner

    N = pos.shape[0]
    exp_pos, outcell, _ = expand_pbc(pos, cell, [True, True, True], CUTOFF)
    g = radius_graph(pos, exp_pos, torch.tensor([0, N]), torch.tensor([0, exp_pos.shape[0]]), CUTOFF, 1e-4, None)
    W, Wi = node_wigner(pos)
    We, Wie = node_wigner(exp_pos)
    smear = GaussianSmearing(NB, cutoff=CUTOFF).to(dev)
    rbf = smear(g["f_dist"]) if materialize_rbf else smear
    bd = dict(g)
    bd.update({"f_outcell_index": outcell, "f_exp_node_pos": exp_pos, "wigner": W, "wigner_inv": Wi,
               "wigner_exp": We, "wigner_inv_exp": Wie})
    return bd, rbf


def layer_step(layer, pos, x, Z, bd, rbf, dout, leaves):
    out, _ = layer(node_pos=pos, node_irreps_input=x, edge_dis=bd["f_dist"], edge_vec=bd["f_edge_vec"],
                   attn_weight=rbf, atomic_numbers=Z, poly_dist=bd["f_poly_dist"], batched_data=bd)
    grads = torch.autograd.grad(out, leaves, dout, allow_unused=True)
    return out, grads


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    def __init__(self, index):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None
        # nvidia-smi takes about a second to print its first sample: wait for it (bounded) so that a
        # short timed region still gets samples, and count only the samples taken after this point
        self.skip = 0
        t_end = time.time() + 5.0
        while self.p is not None and time.time() < t_end:
            with open(self.f.name) as fh:
                n = sum(1 for r in fh if r.strip())
            if n:
                self.skip = n
                break
            time.sleep(0.05)

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        rows = rows[self.skip:] or rows[-1:]   # at least the last sample before the region ended
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) >= 9 and r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in rows:
            if len(r) >= 9:
                for nme, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(nme)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# whether the timed span kept its q.k scores for the backward (the model's and the layer's default at
# 128 heads of 8): the forward then also writes them and the softmax backward reads them instead of q
SPAN_LOGITS_KEPT = True


def fwd_algorithmic_bytes(N, N2, E):
    """Compulsory bytes of one e2a_attn_fwd launch (fp32): q, k, value rows, gate+inputhead, poly, dist,
    col, row_ptr read once; out, beta, row stats (and the kept q.k scores) written once."""
    HD, CH = HEADS * DHEAD, 58 * HEADS
    kept = E * HEADS if SPAN_LOGITS_KEPT else 0
    return 4 * (N * HD + N2 * HD + N2 * CH + E * 2 * HEADS + E * 3 + (N + 1) + N * CH + E * HEADS + 2 * N * HEADS
                + kept)


def bwdq_algorithmic_bytes(N, N2, E):
    HD, CH = HEADS * DHEAD, 58 * HEADS
    reads = N * HD + N2 * HD + N2 * CH + E * 2 * HEADS + E * 3 + (N + 1) + E * HEADS + 2 * N * HEADS + N * CH
    writes = N * HD + E * 2 * HEADS + 2 * E + E * HEADS
    return 4 * (reads + writes)


def bwdk_algorithmic_bytes(N, N2, E):
    HD, CH = HEADS * DHEAD, 58 * HEADS
    reads = N * HD + N * CH + E * HEADS * 2 + 2 * E + (N2 + 1)
    writes = N2 * HD + N2 * CH
    return 4 * (reads + writes)


# dram__bytes_read.sum + dram__bytes_write.sum per launch of a span entry point (sum over its kernels),
# from one ncu capture of a small case (the 20k-atom layer: 640,210 edges; profiles/attn_kernels_20k_full.md)
# scaled to a full launch by the edges processed (nodes, keys and edges grow together at a fixed
# neighbour count): e2a_attn_fwd 4.547 GB and e2a_attn_bwd_value 3.352 GB at 20k atoms.  The softmax
# backward and d_k entry points were not in that capture (None).
_TRAFFIC_20K = {"e2a_attn_fwd": 4.547e9, "e2a_attn_bwd_value": 3.352e9}
_E_20K = 640210
MEASURED_TRAFFIC_DEFAULT = {k: v * 3197986 / _E_20K for k, v in _TRAFFIC_20K.items()}   # layer workload
MEASURED_TRAFFIC_MODEL = {k: v * 3131680 / _E_20K for k, v in _TRAFFIC_20K.items()}     # model workload


def bwdv_algorithmic_bytes(N, N2, E):
    """e2a_attn_bwd_value: own value row and each cotangent row once, beta, key CSR; d_value, d_beta."""
    CH = 58 * HEADS
    return 4 * (N2 * CH + N * CH + E * HEADS + 2 * E + N2 + 1 + N2 * CH + E * HEADS)


def bwds_algorithmic_bytes(N, N2, E):
    """e2a_attn_bwd_softmax: q (or the kept q.k scores), k rows once, gate + inputhead, poly, dist, col,
    row_ptr, d_beta, row stats; d_gate + d_inputhead, d_poly, d_dist, ds, d_q."""
    HD = HEADS * DHEAD
    qs = E * HEADS if SPAN_LOGITS_KEPT else N * HD
    reads = qs + N2 * HD + E * 2 * HEADS + 3 * E + N + 1 + E * HEADS + 2 * N * HEADS
    writes = E * 2 * HEADS + 2 * E + E * HEADS + N * HD
    return 4 * (reads + writes)


def bwddk_algorithmic_bytes(N, N2, E):
    """e2a_attn_bwd_dk: q rows once, ds, key CSR; d_k."""
    HD = HEADS * DHEAD
    return 4 * (N * HD + E * HEADS + N2 + 1 + 2 * E + N2 * HD)


# ------------------------------------------------------------------------------------------------
def cpu_baseline_setup(n_atoms, k):
    """Build the CPU oracle of the layer (reference algorithm restated) on a bounded sample and
    return a closure running one forward + backward on all host threads."""
    from oracle import attention_ref as R
    from oracle import graph_ref
    from ubio_molfm_b200.graph import pbc_image_offsets
    from ubio_molfm_b200.nn import GaussianSmearing, polynomial
    from ubio_molfm_b200.synthetic import uniform_box
    from ubio_molfm_b200.wigner import node_wigner

    torch.set_num_threads(os.cpu_count() or 1)
    pos, Z, cell = uniform_box(n_atoms, k, CUTOFF, seed=7)
    pos = pos.astype(np.float32)
    off = pbc_image_offsets(cell, [True] * 3, CUTOFF).numpy()
    ia = graph_ref.pbc_expand(pos, off, CUTOFF)
    outcell = ia % n_atoms
    exp_pos = (pos[outcell] + off[ia // n_atoms]).astype(np.float32)
    qi, ni, d = graph_ref.radius_graph(pos, exp_pos, [0, n_atoms], [0, len(exp_pos)], CUTOFF, 1e-4, None)
    layer = make_layer("cpu")
    p = {kk: v.detach() for kk, v in layer.state_dict().items()}
    g = torch.Generator().manual_seed(1)
    x = torch.randn(n_atoms, 9, C_CH, generator=g, requires_grad=True)
    dout = torch.randn(n_atoms, 9, C_CH, generator=g)
    Zt = torch.tensor(Z)

    def run():
        pos_t = torch.tensor(pos, requires_grad=True)
        exp_t = torch.tensor(exp_pos, requires_grad=True)
        dist = torch.tensor(d, requires_grad=True)
        W, Wi = node_wigner(pos_t)
        We, Wie = node_wigner(exp_t)
        poly = polynomial(dist, CUTOFF)
        rbf = GaussianSmearing(NB, cutoff=CUTOFF)(dist)
        bd = {"query_idx": torch.tensor(qi), "neighbor_idx": torch.tensor(ni),
              "f_outcell_index": torch.tensor(outcell), "f_exp_node_pos": exp_t, "wigner": W, "wigner_inv": Wi,
              "wigner_exp": We, "wigner_inv_exp": Wie}
        out = R.attention_layer(p, HEADS, DHEAD, pos_t, x, dist, rbf, Zt, poly, bd)
        torch.autograd.grad(out, [x, pos_t, exp_t, dist], dout)

    desc = (f"{n_atoms} atoms, {len(qi)} edges: 1 layer fwd+bwd of the CPU oracle (the reference's "
            f"pure-PyTorch attention path restated), fp32")
    return run, desc


def run_cpu_baseline(n_atoms, k, steps=1, warmup=0):
    run, desc = cpu_baseline_setup(n_atoms, k)
    for _ in range(warmup):
        run()
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": n_atoms / t, "unit": "atom-steps/s", "cores": torch.get_num_threads(), "kind": kind,
            "sample": f"{desc}; median of {steps} steps, {t:.2f} s/step", "cpu_model": _cpu_model()}


def _cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


# ------------------------------------------------------------------------------------------------
def run_reference(args, ws, rank):
    if rank != 0:
        return
    n = args.cpu_atoms or 1500
    cb = run_cpu_baseline(n, args.k, args.steps, min(args.warmup, 1))
    v = cb["value"]
    line = {"impl": "reference", "metric": "atom-steps/s", "value": v, "unit": "atom-steps/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * n / v,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded uniform periodic box, seeded random weights)",
            "config": config_dict(args, extra={"reference_sample_atoms": n}),
            "cpu_baseline": cb,
            "e2e": {"value": v, "unit": "atom-steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def run_ours(args, ws, rank, local):
    from ubio_molfm_b200 import _lib, ops
    from ubio_molfm_b200.synthetic import uniform_box

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    layer = make_layer(dev)
    pos_np, Z_np, cell = uniform_box(args.atoms, args.k, CUTOFF, seed=100 + rank)
    pos = torch.tensor(pos_np, dtype=torch.float32, device=dev)
    Z = torch.tensor(Z_np, device=dev)
    chunked = bool(args.edge_chunk)
    bd, rbf = build_inputs(pos, Z, cell, dev, layer, materialize_rbf=not chunked)
    N, N2, E = args.atoms, bd["f_outcell_index"].shape[0], bd["query_idx"].numel()
    g = torch.Generator(device=dev).manual_seed(rank)
    x = torch.randn(N, 9, C_CH, device=dev, generator=g)
    dout = torch.randn(N, 9, C_CH, device=dev, generator=g)
    # leaves: everything the forces chain differentiates through
    base = {"x": x, "pos": pos, "f_dist": bd["f_dist"], "poly": bd["f_poly_dist"], "exp": bd["f_exp_node_pos"],
            "W": bd["wigner"], "Wi": bd["wigner_inv"], "We": bd["wigner_exp"], "Wie": bd["wigner_inv_exp"]}
    if not chunked:
        base["rbf"] = rbf
    leaf = {k: v.detach().requires_grad_(True) for k, v in base.items()}
    bdl = dict(bd)
    bdl.update({"f_dist": leaf["f_dist"], "f_poly_dist": leaf["poly"], "f_exp_node_pos": leaf["exp"],
                "wigner": leaf["W"], "wigner_inv": leaf["Wi"], "wigner_exp": leaf["We"], "wigner_inv_exp": leaf["Wie"]})
    leaves = list(leaf.values())
    if chunked:
        from ubio_molfm_b200.nn import RbfSpec
        # the memory mode: edge side in checkpointed row blocks, Q / K projections formed again in the backward
        layer.edge_chunk = args.edge_chunk
        layer.query_linear.recompute_pair_product = True
        layer.key_linear.recompute_pair_product = True

    def step():
        aw = RbfSpec(leaf["f_dist"], rbf.offset, rbf.coeff) if chunked else leaf["rbf"]
        return layer_step(layer, leaf["pos"], leaf["x"], Z, bdl, aw, dout, leaves)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    ops.TIMER.enabled = True
    ops.TIMER.events = {}
    launches0 = _lib.launch_count()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    ops.TIMER.enabled = False
    launches_timed = _lib.launch_count() - launches0
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / args.steps
    ms = max_over_ranks(ms, ws, dev)
    kern = ops.TIMER.summary()
    # dominant kernel of this package
    top = max(kern.items(), key=lambda kv: kv[1][1])
    name, (nl, tot) = top
    alg = {"e2a_attn_fwd": fwd_algorithmic_bytes, "e2a_attn_bwd_query": bwdq_algorithmic_bytes,
           "e2a_attn_bwd_key": bwdk_algorithmic_bytes, "e2a_attn_bwd_value": bwdv_algorithmic_bytes,
           "e2a_attn_bwd_softmax": bwds_algorithmic_bytes, "e2a_attn_bwd_dk": bwddk_algorithmic_bytes}[name](N, N2, E)
    # in row blocks each launch covers one block: its share of the graph's bytes (the key-table term split
    # evenly, which undercounts the key rows a block reads)
    blocks = len(layer._edge_chunks(dict(bdl), N) or [None]) if chunked else 1
    alg = alg / blocks
    per_launch_ms = tot / nl
    peak, peak_kind = measured_peaks()
    achieved = alg / (per_launch_ms * 1e-3) / 1e9
    roof = {"kernel": name, "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "peak_source": peak_kind,
            "traffic": (MEASURED_TRAFFIC_DEFAULT.get(name)
                        if (args.atoms, args.k) == (100_000, 32) and not chunked else None),
            "algorithmic_bytes_per_launch": alg, "launch_ms": round(per_launch_ms, 4), "edge_blocks": blocks,
            "kernels_ms_per_launch": {k: round(v[1] / v[0], 4) for k, v in kern.items()},
            "step_share": {k: round(v[1] / args.steps / ms, 4) for k, v in kern.items()}}
    value = ws * N * 1e3 / ms

    # ---------------- e2e through the public API from pinned host buffers ----------------
    e2e = None
    if not args.no_e2e:
        del leaf, bdl, leaves, bd, rbf
        torch.cuda.empty_cache()
        h_pos = torch.tensor(pos_np, dtype=torch.float32).pin_memory()
        h_Z = torch.tensor(Z_np).pin_memory()
        h_x = x.cpu().pin_memory()
        h_dout = dout.cpu().pin_memory()
        h_out = torch.empty((N, 9, C_CH), dtype=torch.float32).pin_memory()
        h_dx = torch.empty_like(h_out).pin_memory()
        h_dpos = torch.empty((N, 3), dtype=torch.float32).pin_memory()

        def e2e_step():
            p = h_pos.to(dev, non_blocking=True).requires_grad_(True)
            z = h_Z.to(dev, non_blocking=True)
            xx = h_x.to(dev, non_blocking=True).requires_grad_(True)
            do = h_dout.to(dev, non_blocking=True)
            b, r = build_inputs(p, z, cell, dev, layer, materialize_rbf=not chunked)
            if chunked:
                r = RbfSpec(b["f_dist"], r.offset, r.coeff)
            out, (gx, gp) = layer_step(layer, p, xx, z, b, r, do, [xx, p])
            h_out.copy_(out.detach(), non_blocking=True)
            h_dx.copy_(gx, non_blocking=True)
            h_dpos.copy_(gp, non_blocking=True)

        for _ in range(max(1, args.warmup)):
            e2e_step()
        torch.cuda.synchronize()
        barrier(ws)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            e2e_step()
        e1.record()
        torch.cuda.synchronize()
        barrier(ws)
        ems = max_over_ranks(e0.elapsed_time(e1) / args.steps, ws, dev)
        h2d = h_pos.numel() * 4 + h_Z.numel() * 8 + h_x.numel() * 4 + h_dout.numel() * 4
        d2h = h_out.numel() * 4 + h_dx.numel() * 4 + h_dpos.numel() * 4
        e2e = {"value": ws * N * 1e3 / ems, "unit": "atom-steps/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": round(ems, 3),
               "includes": "H2D, PBC images, radius graph + CSR, Wigner, RBF, layer fwd+bwd, D2H"}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        cpu = run_cpu_baseline(args.cpu_atoms or 1500, args.k, 1, 0)

    if rank == 0:
        line = {"metric": "atom-steps/s", "value": round(value, 1), "unit": "atom-steps/s", "n_gpus": ws,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded uniform periodic box, seeded random weights)",
                "config": config_dict(args, E, N2), "roofline": roof, "cpu_baseline": cpu, "e2e": e2e,
                "gpu_launches": launches_timed, "clocks": clk,
                "peak_memory_gb": round(torch.cuda.max_memory_allocated(dev) / 1e9, 1)}
        print(json.dumps(line))


# ------------------------------------------------------------------------------------------------
# Full energy + forces workload
# ------------------------------------------------------------------------------------------------
MODEL_CFG = dict(irreps_node_embedding=f"{C_CH}x0e+{C_CH}x1e+{C_CH}x2e", num_layers=4, max_neighbors=32,
                 max_radius=CUTOFF, number_of_basis=NB, num_attn_heads=HEADS, attn_scalar_head=DHEAD,
                 irreps_head=HEAD_IRREPS, norm_layer="rms_norm_sh", alpha_drop=0.0, avg_degree=23.01)


def model_config_dict(args, N=None, E=None, N2=None, extra=None):
    d = {"workload": "E2Former-V2 energy+forces (full-size backbone, 4 layers) on a ~1e5-atom periodic "
                     "system: 8,000-atom H/C/N/O/S blob in rigid water, 100 A cube, cutoff 6 A, <= 32 neighbours",
         "layers": 4, "irreps": MODEL_CFG["irreps_node_embedding"], "heads": HEADS, "attn_scalar_head": DHEAD,
         "irreps_head": HEAD_IRREPS, "rbf": NB, "cutoff": CUTOFF, "max_neighbors": 32,
         "l2": "inputs larger than L2 (value rows alone are GBs per layer)", "parallelism": f"replicas x{args.gpus}",
         "graph": "rebuilt every step (PBC images, radius graph, CSR)"}
    if N is not None:
        d.update({"atoms_per_rank": N, "edges_per_rank": E, "expanded_nodes_per_rank": N2})
    if extra:
        d.update(extra)
    return d


def make_model(dev, seed=0):
    from ubio_molfm_b200.model import E2FormerPotential
    from ubio_molfm_b200.synthetic import seeded_params_

    m = E2FormerPotential(**MODEL_CFG)
    seeded_params_(m, seed)
    return m.to(dev).eval()


def cpu_model_setup(n_atoms):
    """The CPU oracle of the full energy + forces evaluation on a bounded sample (an ``n_atoms``
    biomolecular box at the model's cutoff and neighbour cap); returns a closure and a description."""
    from oracle import graph_ref
    from oracle import model_ref as M
    from ubio_molfm_b200.graph import pbc_image_offsets
    from ubio_molfm_b200.synthetic import bio_box

    torch.set_num_threads(os.cpu_count() or 1)
    m = make_model("cpu")
    p = {k: v.detach() for k, v in m.decoder.state_dict().items()}
    ph = {k: v.detach() for k, v in m.energy_head.state_dict().items()}
    pos, Z, cell = bio_box(n_atoms, seed=3)
    pos = pos.astype(np.float32)
    off = pbc_image_offsets(cell, [True] * 3, CUTOFF).numpy()
    ia = graph_ref.pbc_expand(pos, off, CUTOFF)
    oc, offs = ia % n_atoms, off[ia // n_atoms]
    exp = (pos[oc] + offs).astype(np.float32)
    qi, ni, _ = graph_ref.radius_graph(pos, exp, [0, n_atoms], [0, len(exp)], CUTOFF, 1e-4, 32)
    graph = (torch.tensor(qi), torch.tensor(ni), torch.tensor(oc), torch.tensor(offs), True)
    pos_t, Z_t = torch.tensor(pos), torch.tensor(Z)

    def run():
        M.energy_forces(p, ph, MODEL_CFG, pos_t, Z_t, graph)

    desc = (f"{n_atoms}-atom biomolecular box, {len(qi)} edges: energy+forces of the full-size model by the "
            f"CPU oracle (the reference's pure-PyTorch path restated), fp32")
    return run, desc


def cpu_model_setup_reference(n_atoms):
    """The reference's own CPU path on the same bounded sample: its unmodified ``E2FormerBackbone``
    (PBC expansion, dense radius graph, E2former, charge / multiplicity embedding) and
    ``MLP_energy_head`` from the offline install under baseline/_ref, imported through the test-only
    shim that stands in for its missing third-party packages (e3nn, torch_geometric, faiss), energy
    and forces = -dE/dpos by autograd.  Returns (closure, description) or (None, why)."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "molfm")):
        return None, "the reference is not installed under baseline/_ref"
    os.environ["E2A_REFERENCE_ROOT"] = ref
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    try:
        import importlib

        import refshim

        from ubio_molfm_b200.synthetic import bio_box, seeded_params_

        refshim.load_reference()
        wrapper = importlib.import_module("molfm.models.e2former.e2former_wrapper")
        head_mod = importlib.import_module("molfm.pipeline.head")
    except Exception as exc:  # noqa: BLE001
        return None, f"the reference did not import: {exc!r}"[:300]
    torch.set_num_threads(os.cpu_count() or 1)
    bb = wrapper.E2FormerBackbone(use_faiss=False, encoder="default", tp_type="QK_alpha", attn_type="so2-first-order",
                                  **MODEL_CFG).eval()
    seeded_params_(bb, 0)
    head = head_mod.MLP_energy_head(C_CH, 2)
    seeded_params_(head, 1)
    pos, Z, cell = bio_box(n_atoms, seed=3)
    P = torch.tensor(pos, dtype=torch.float32).unsqueeze(0)
    Zt = torch.tensor(Z, dtype=torch.long).unsqueeze(0)

    def run():
        p = P.clone().requires_grad_(True)
        bd = {"pos": p, "atom_masks": torch.ones_like(Zt, dtype=torch.bool), "atomic_numbers": Zt,
              "pbc": torch.ones((1, 3), dtype=torch.int32), "cell": torch.tensor(cell, dtype=torch.float32)[None],
              "charge": torch.zeros((1, 1), dtype=torch.int32), "multiplicity": torch.ones((1, 1), dtype=torch.int32)}
        out = bb(bd)
        e = head(out["node_featuresBxN"], out["node_irrepsBxN"]).sum()
        torch.autograd.grad(e, p)

    desc = (f"{n_atoms}-atom biomolecular box: energy+forces of the full-size model by the reference's own "
            f"E2FormerBackbone + MLP_energy_head on the CPU (pure-PyTorch path, fp32)")
    return run, desc


def run_cpu_model(n_atoms, steps=1, warmup=0):
    run, desc = cpu_model_setup_reference(n_atoms)
    kind = "reference"
    if run is None:
        why = desc
        run, desc = cpu_model_setup(n_atoms)
        kind = "port"
        desc = f"{desc} (the reference itself: {why})"
    for _ in range(warmup):
        run()
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": n_atoms / t, "unit": "atom-steps/s", "cores": torch.get_num_threads(), "kind": kind,
            "sample": f"{desc}; median of {steps} steps, {t:.2f} s/step", "cpu_model": _cpu_model()}


def run_reference_model(args, ws, rank):
    if rank != 0:
        return
    n = args.cpu_atoms or 500
    cb = run_cpu_model(n, args.steps, min(args.warmup, 1))
    v = cb["value"]
    line = {"impl": "reference", "metric": "atom-steps/s", "value": v, "unit": "atom-steps/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * n / v, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded periodic systems, seeded random weights)",
            "config": model_config_dict(args, extra={"reference_sample_atoms": n}), "cpu_baseline": cb,
            "e2e": {"value": v, "unit": "atom-steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def run_model(args, ws, rank, local):
    from ubio_molfm_b200 import _lib, ops
    from ubio_molfm_b200.synthetic import blob_in_water

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    from ubio_molfm_b200 import linear as _linear

    _linear.PASSES = 1 if args.projections == "tf32" else 3
    model = make_model(dev)
    pos_np, Z_np, cell_np = blob_in_water(seed=100 if (ws > 1 and not args.replicas) else 100 + rank)
    pos = torch.tensor(pos_np, dtype=torch.float32, device=dev)
    Z = torch.tensor(Z_np, device=dev)
    cell = torch.tensor(cell_np, dtype=torch.float32)
    pbc = (True, True, True)
    N = pos.shape[0]
    g, _ = model.build_graph(pos, cell, pbc, None)
    E, N2 = g["query_idx"].numel(), g["f_exp_node_pos"].shape[0]
    del g

    domain = ws > 1 and not args.replicas
    from ubio_molfm_b200 import linear
    from ubio_molfm_b200.domain import HALO_STATS
    if domain:
        from ubio_molfm_b200.domain import domain_energy_forces

        def step():
            return domain_energy_forces(model, pos, Z, cell, pbc)
    else:
        def step():
            return model(pos, Z, cell, pbc)

    for _ in range(args.warmup):
        step()
    global SPAN_LOGITS_KEPT
    SPAN_LOGITS_KEPT = bool(model.decoder.blocks[0].ga.keep_logits)
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    ops.TIMER.enabled = True
    ops.TIMER.events = {}
    linear.GEMM_TIMER.enabled = True
    linear.GEMM_TIMER.records = []
    if domain:
        HALO_STATS.enabled = True
        HALO_STATS.records = []
    launches0 = _lib.launch_count()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    ops.TIMER.enabled = False
    linear.GEMM_TIMER.enabled = False
    HALO_STATS.enabled = False
    launches_timed = _lib.launch_count() - launches0
    clk = clocks.stop()
    ms = max_over_ranks(t0.elapsed_time(t1) / args.steps, ws, dev)
    kern = ops.TIMER.summary()
    g_n, g_ms, g_flop = linear.GEMM_TIMER.summary()
    halo = HALO_STATS.summary() if domain else None
    name, (nl, tot) = max(kern.items(), key=lambda kv: kv[1][1])
    if domain:   # this rank's share of the span: its owned rows, their edges, their expanded keys
        from ubio_molfm_b200.domain import domain_graph
        _, _, local_gid, geom = domain_graph(pos, cell, pbc, CUTOFF, 32, ws, rank)
        N_r, E_r, N2_r = local_gid.numel(), geom["query_idx"].numel(), geom["outcell"].numel()
    else:
        N_r, E_r, N2_r = N, E, N2
    alg = {"e2a_attn_fwd": fwd_algorithmic_bytes, "e2a_attn_bwd_query": bwdq_algorithmic_bytes,
           "e2a_attn_bwd_key": bwdk_algorithmic_bytes, "e2a_attn_bwd_value": bwdv_algorithmic_bytes,
           "e2a_attn_bwd_softmax": bwds_algorithmic_bytes, "e2a_attn_bwd_dk": bwddk_algorithmic_bytes}[name](N_r, N2_r, E_r)
    per_launch_ms = tot / nl
    peak, peak_kind = measured_peaks()
    achieved = alg / (per_launch_ms * 1e-3) / 1e9
    roof = {"kernel": name, "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "peak_source": peak_kind,
            "traffic": None if domain else MEASURED_TRAFFIC_MODEL.get(name),
            "algorithmic_bytes_per_launch": alg, "launch_ms": round(per_launch_ms, 4),
            "kernels_ms_per_launch": {k: round(v[1] / v[0], 4) for k, v in kern.items()},
            "step_share": {k: round(v[1] / args.steps / ms, 4) for k, v in kern.items()}}
    # every span entry point against its algorithmic bytes, and the tensor-core projections of the step
    entries = {}
    for k, (nl_k, tot_k) in kern.items():
        fn = {"e2a_attn_fwd": fwd_algorithmic_bytes, "e2a_attn_bwd_value": bwdv_algorithmic_bytes,
              "e2a_attn_bwd_softmax": bwds_algorithmic_bytes, "e2a_attn_bwd_dk": bwddk_algorithmic_bytes,
              "e2a_attn_bwd_query": bwdq_algorithmic_bytes, "e2a_attn_bwd_key": bwdk_algorithmic_bytes}.get(k)
        if fn is None:
            continue
        b_k = fn(N_r, N2_r, E_r)
        ms_k = tot_k / nl_k
        entries[k] = {"ms": round(ms_k, 4), "algorithmic_bytes": b_k,
                      "frac": round(b_k / (ms_k * 1e-3) / 1e9 / peak, 4)}
    roof["entry_points"] = entries
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            bf16s = float(json.load(f)["bf16_tflops_sustained"])
        bsrc = "measured"
    except Exception:
        bf16s, bsrc = 1400.0, "fallback"
    if g_n:
        tfs = g_flop / args.steps / (g_ms / args.steps * 1e-3) / 1e12
        passes = 1 if args.projections == "tf32" else 3
        roof["gemm"] = {"kernel": f"k_gemm_ws (tcgen05 {passes}xTF32)", "bound": "tensor",
                        "launches_per_step": g_n // args.steps,
                        "ms_per_step": round(g_ms / args.steps, 3), "tflop_per_step": round(g_flop / args.steps / 1e12, 3),
                        "achieved": round(tfs, 1), "unit": "TFLOP/s of fp32-accurate output",
                        "ceiling": f"{passes}xTF32: the tf32 rate (half the measured bf16 rate) / {passes}",
                        "ceiling_tflops": round(bf16s / 2 / passes, 1),
                        "frac_of_ceiling": round(tfs / (bf16s / 2 / passes), 3),
                        "peak_bf16_sustained": bf16s, "frac_of_bf16_sustained": round(tfs / bf16s, 4),
                        "peak_source": bsrc, "step_share": round(g_ms / args.steps / ms, 4),
                        "note": "NxTF32 issues N tf32 MMAs per product",
                        "by_shape_MNK_launches_ms_tflops": linear.GEMM_TIMER.by_shape()}
    value = (1 if domain else ws) * N * 1e3 / ms

    e2e = None
    if not args.no_e2e:
        h_pos = torch.tensor(pos_np, dtype=torch.float32).pin_memory()
        h_Z = torch.tensor(Z_np).pin_memory()
        h_e = torch.empty(1, dtype=torch.float32).pin_memory()
        h_f = torch.empty((N, 3), dtype=torch.float32).pin_memory()

        def e2e_step():
            p = h_pos.to(dev, non_blocking=True)
            z = h_Z.to(dev, non_blocking=True)
            if domain:
                e, _, f = domain_energy_forces(model, p, z, cell, pbc)
                h_e.copy_(e, non_blocking=True)
                h_f[: f.shape[0]].copy_(f, non_blocking=True)
            else:
                e, f = model(p, z, cell, pbc)
                h_e.copy_(e, non_blocking=True)
                h_f.copy_(f, non_blocking=True)

        for _ in range(max(1, min(args.warmup, 2))):
            e2e_step()
        torch.cuda.synchronize()
        barrier(ws)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            e2e_step()
        e1.record()
        torch.cuda.synchronize()
        barrier(ws)
        ems = max_over_ranks(e0.elapsed_time(e1) / args.steps, ws, dev)
        e2e = {"value": (1 if domain else ws) * N * 1e3 / ems, "unit": "atom-steps/s",
               "h2d_bytes_per_step": h_pos.numel() * 4 + h_Z.numel() * 8,
               "d2h_bytes_per_step": h_e.numel() * 4 + h_f.numel() * 4, "ms_per_step": round(ems, 3),
               "includes": "H2D positions + atomic numbers, PBC images, radius graph + CSR, Wigner, backbone, "
                           "energy head, forces, D2H energy + forces"}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        cpu = run_cpu_model(args.cpu_atoms or 500, 1, 1)

    if rank == 0:
        cfgd = model_config_dict(args, N, E, N2)
        if domain:
            cfgd["parallelism"] = f"slab domain decomposition x{ws}, per-layer halo exchange (NCCL all_to_all)"
            cfgd.update({"atoms_total": N, "edges_total": E, "atoms_per_rank": round(N / ws),
                         "rank0_local_atoms_incl_ghosts": N_r, "rank0_edges": E_r, "rank0_expanded_nodes": N2_r})
            for k in ("edges_per_rank", "expanded_nodes_per_rank"):
                cfgd.pop(k, None)
        line = {"metric": "atom-steps/s", "value": round(value, 1), "unit": "atom-steps/s", "n_gpus": ws,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
                "scaling": "strong" if domain else "weak", "vs_baseline": None,
                "dtype": "f32" if args.projections == "fp32" else "f32 (tf32 projections)",
                "data": "synthetic (seeded blob-in-water periodic system, seeded random weights)",
                "config": cfgd, "roofline": roof, "cpu_baseline": cpu, "e2e": e2e,
                "gpu_launches": launches_timed, "clocks": clk,
                "peak_memory_gb": round(torch.cuda.max_memory_allocated(dev) / 1e9, 1)}
        if halo is not None:
            line["halo_exchange"] = {d: {"calls_per_step": v["calls"] // args.steps,
                                         "ms_per_step": round(v["ms"] / args.steps, 3),
                                         "bytes_per_step": v["bytes"] // args.steps} for d, v in halo.items()}
        print(json.dumps(line))


def run_molecules(args, ws, rank, local):
    """Config 4: a batch of non-periodic molecules (10-60 atoms, charges in [-1, 1], multiplicity 1)
    sharded across ranks by size; each rank evaluates its molecules' energies and forces (batched,
    systems independent, each with its charge embedding); energies and forces gathered to rank 0.  The full-size backbone at the reference's small-molecule cutoff (4.5 A, <= 32 neighbours)."""
    from ubio_molfm_b200 import _lib
    from ubio_molfm_b200.domain import gather_molecule_results, molecules_energy_forces, shard_molecules
    from ubio_molfm_b200.model import E2FormerPotential
    from ubio_molfm_b200.synthetic import molecule_batch, seeded_params_

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    torch.backends.cuda.matmul.allow_tf32 = False
    m = E2FormerPotential(**dict(MODEL_CFG, max_radius=4.5))
    seeded_params_(m, 0)
    m = m.to(dev).eval()
    mols = molecule_batch(args.molecules, 10, 60, seed=11)
    parts = shard_molecules([len(z) for _, z, _, _ in mols], ws)
    mine = parts[rank]
    my = [mols[i] for i in mine]           # (pos, Z, charge, multiplicity)
    n_atoms_total = sum(len(z) for _, z, _, _ in mols)

    def step():
        e, f = molecules_energy_forces(m, my, dev)
        if ws > 1:
            e, f = gather_molecule_results(e, f, mine, len(mols))
        if rank == 0:   # the results reach the host on rank 0
            e = e.cpu()
            torch.cat(f).cpu()
        return e

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(ws)
    clocks = ClockSampler(local)
    launches0 = _lib.launch_count()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    barrier(ws)
    clk = clocks.stop()
    launches = _lib.launch_count() - launches0
    ms = max_over_ranks(t0.elapsed_time(t1) / args.steps, ws, dev)
    if rank == 0:
        h2d = sum(len(m[1]) * (12 + 8) for m in my)
        line = {"metric": "atom-steps/s", "value": round(n_atoms_total * 1e3 / ms, 1), "unit": "atom-steps/s",
                "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded random-tree molecules, seeded random weights)",
                "config": {"workload": f"energy+forces of {len(mols)} non-periodic molecules (10-60 atoms, "
                                       f"H/C/N/O/F/S/Cl), full-size backbone, cutoff 4.5 A, <= 32 neighbours",
                           "molecules": len(mols), "atoms_total": n_atoms_total,
                           "molecules_per_s": round(len(mols) * 1e3 / ms, 1),
                           "parallelism": f"molecules sharded by size over {ws} ranks; energies and forces gathered to rank 0",
                           "l2": "inputs larger than L2"},
                "e2e": {"value": round(n_atoms_total * 1e3 / ms, 1), "unit": "atom-steps/s",
                        "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4 * len(mols) + 12 * n_atoms_total,
                        "includes": "the timed step copies every batch's positions / types from host memory and, on rank 0, all energies and forces back"},
                "gpu_launches": launches, "clocks": clk}
        print(json.dumps(line))


# ------------------------------------------------------------------------------------------------
# Same-box kernel bar: this package's attention span against the reference's own Triton kernels
# ------------------------------------------------------------------------------------------------
def _load_reference_triton():
    """The reference's Triton modules (triton_dr/*.py) from the offline install under baseline/_ref,
    loaded without executing the parent packages' __init__ (they import e3nn / torch_geometric)."""
    import importlib
    import types

    base = os.path.join(ROOT, "baseline", "_ref", "molfm", "models", "e2former")
    if not os.path.isdir(os.path.join(base, "triton_dr")):
        return None, "the reference is not installed under baseline/_ref"
    for name, path in [("molfm", os.path.join(ROOT, "baseline", "_ref", "molfm")),
                       ("molfm.models", os.path.join(ROOT, "baseline", "_ref", "molfm", "models")),
                       ("molfm.models.e2former", base)]:
        if name not in sys.modules:
            m = types.ModuleType(name)
            m.__path__ = [path]
            sys.modules[name] = m
    try:
        mods = {s: importlib.import_module(f"molfm.models.e2former.triton_dr.{s}") for s in
                ("triton_sparse_qk_autograd", "sparse_alpha_sum_edge_index_autograd",
                 "sparse_v_agg_edge_index_cblocked_bench")}
    except Exception as exc:  # noqa: BLE001
        return None, f"reference Triton kernels failed to import: {exc!r}"[:300]
    return mods, None


def reference_span(mods, q, k, v, gi, poly, dist, q_idx, n_idx, md, N):
    """The reference's attention span on its Triton path, composed as E2AttentionArbOrder_sparse
    does (e2former.py:311-364 and 393-422; so2_tensor_product.py:341-389 aggregates the merged value
    with one call): Triton q.k, torch segmented max / exp, Triton row sum, alpha / r, Triton V
    aggregation."""
    H = q.shape[1]
    qk = mods["triton_sparse_qk_autograd"].sparse_qk_edge_index_triton(q, k, q_idx, n_idx, metadata=md)
    gate, inputhead = gi[:, :H], gi[:, H:]
    alpha = gate * qk
    qil = q_idx.long()
    idx = qil.unsqueeze(-1).expand(-1, H)
    amax = torch.full((N, H), -torch.inf, device=q.device, dtype=alpha.dtype)
    amax.scatter_reduce_(0, idx, alpha, reduce="amax", include_self=True)
    alpha = torch.exp(alpha - amax[qil]) * poly.unsqueeze(-1)
    asum = mods["sparse_alpha_sum_edge_index_autograd"].sparse_alpha_sum_edge_index_triton(
        alpha, q_idx, N, metadata=(md[0], md[2]))
    alpha = alpha * inputhead / (asum[qil] + 1e-3)
    alpha_r = alpha / dist.unsqueeze(-1).clamp_min(1e-6)
    return mods["sparse_v_agg_edge_index_cblocked_bench"].sparse_v_agg_edge_index_triton_cblocked(
        value=v.contiguous(), alpha=alpha_r, query_index=q_idx, value_index=n_idx, num_queries=N, metadata=md)


def compare_kernel_functions(mods, ins, q_idx, n_idx, md_ref, md_ours, N, N2, timed, dev):
    """Each kernel-level function of the reference (triton_dr/*.py) against this package's function of
    the same name and signature (``ubio_molfm_b200.ops``) on the same inputs: forward, and forward +
    backward with a seeded cotangent; ms (median) and the largest relative difference of the outputs."""
    from ubio_molfm_b200 import ops

    H = ins[0].shape[1]
    E = q_idx.numel()
    gen = torch.Generator(device=dev).manual_seed(7)
    qi32, ni32 = q_idx.to(torch.int32), n_idx.to(torch.int32)
    alpha = torch.rand(E, H, device=dev, generator=gen)
    sh = torch.randn(E, 5, device=dev, generator=gen)
    fea = torch.randn(E, 128, device=dev, generator=gen)
    ref_qk = mods["triton_sparse_qk_autograd"].sparse_qk_edge_index_triton
    ref_as = mods["sparse_alpha_sum_edge_index_autograd"].sparse_alpha_sum_edge_index_triton
    ref_va = mods["sparse_v_agg_edge_index_cblocked_bench"].sparse_v_agg_edge_index_triton_cblocked
    import importlib

    ref_eo = importlib.import_module("molfm.models.e2former.triton_dr.edge_degree_outer_autograd").edge_degree_outer_triton
    cases = {
        "sparse_qk_edge_index_triton": (
            lambda f, md, a: f(a[0], a[1], qi32, ni32, metadata=md), [ins[0], ins[1]]),
        "sparse_alpha_sum_edge_index_triton": (
            lambda f, md, a: f(a[0], qi32, N, metadata=(md[0], md[2])), [alpha]),
        "sparse_v_agg_edge_index_triton_cblocked": (
            lambda f, md, a: f(a[0], a[1], qi32, ni32, N, metadata=md), [ins[2], alpha]),
        "edge_degree_outer_triton": (
            lambda f, md, a: f(a[0], a[1], qi32, N, metadata=md), [sh, fea]),
        # bf16 value rows and weights (this package gathers the bf16 rows and sums in fp32)
        "sparse_v_agg_edge_index_triton_cblocked[bf16]": (
            lambda f, md, a: f(a[0], a[1], qi32, ni32, N, metadata=md),
            [ins[2].to(torch.bfloat16), alpha.to(torch.bfloat16)]),
    }
    impls = {"sparse_qk_edge_index_triton": (ref_qk, ops.sparse_qk_edge_index_triton),
             "sparse_alpha_sum_edge_index_triton": (ref_as, ops.sparse_alpha_sum_edge_index_triton),
             "sparse_v_agg_edge_index_triton_cblocked": (ref_va, ops.sparse_v_agg_edge_index_triton_cblocked),
             "edge_degree_outer_triton": (ref_eo, ops.edge_degree_outer_triton),
             "sparse_v_agg_edge_index_triton_cblocked[bf16]": (ref_va, ops.sparse_v_agg_edge_index_triton_cblocked)}
    out = {}
    for name, (call, args) in cases.items():
        row = {}
        for who, fn, md in (("reference", impls[name][0], md_ref), ("ours", impls[name][1], md_ours)):
            leaves = [a.detach().clone().requires_grad_(True) for a in args]
            y = call(fn, md, leaves)
            w = torch.randn(y.shape, device=dev, generator=torch.Generator(device=dev).manual_seed(11))

            def fwd(fn=fn, md=md):
                with torch.no_grad():
                    return call(fn, md, args)

            def fb(fn=fn, md=md, leaves=leaves, w=w):
                return torch.autograd.grad(call(fn, md, leaves), leaves, w)

            row[who] = {"fwd_ms": timed(fwd), "fwd_bwd_ms": timed(fb), "y": y.detach()}
        d = (row["reference"]["y"].float() - row["ours"]["y"].float()).abs().max().item()
        out[name] = {"reference_fwd_ms": row["reference"]["fwd_ms"], "ours_fwd_ms": row["ours"]["fwd_ms"],
                     "reference_fwd_bwd_ms": row["reference"]["fwd_bwd_ms"], "ours_fwd_bwd_ms": row["ours"]["fwd_bwd_ms"],
                     "max_rel_diff": d / max(1.0, row["ours"]["y"].abs().max().item())}
    return out


def run_span(args, ws, rank, local):
    """The attention span alone (q.k, segmented softmax, alpha / r, value aggregation; forward and the
    first-order backward) on the config-2 graph (uniform periodic box, ~k neighbours within 6 A,
    H = 128 heads of 8, C = 58 value rows), this package's kernels against the reference's Triton
    kernels from baseline/_ref on the same inputs, CUDA events, median of ``--steps`` repeats."""
    from ubio_molfm_b200 import _lib, ops
    from ubio_molfm_b200.graph import expand_pbc, radius_graph
    from ubio_molfm_b200.synthetic import uniform_box

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    pos_np, _, cell = uniform_box(args.atoms, args.k, CUTOFF, seed=100)
    pos = torch.tensor(pos_np, dtype=torch.float32, device=dev)
    exp_pos, _, _ = expand_pbc(pos, cell, [True, True, True], CUTOFF)
    N, N2 = pos.shape[0], exp_pos.shape[0]
    g = radius_graph(pos, exp_pos, torch.tensor([0, N]), torch.tensor([0, N2]), CUTOFF, 1e-4, None)
    q_idx, n_idx = g["query_idx"], g["neighbor_idx"]
    E = q_idx.numel()
    H, D, C = HEADS, DHEAD, 58
    gen = torch.Generator(device=dev).manual_seed(0)
    ins = [torch.randn(N, H, D, device=dev, generator=gen) / D ** 0.5, torch.randn(N2, H, D, device=dev, generator=gen),
           torch.randn(N2, C, H, device=dev, generator=gen), torch.randn(E, 2 * H, device=dev, generator=gen),
           g["f_poly_dist"].detach(), g["f_dist"].detach()]
    dout = torch.randn(N, C, H, device=dev, generator=gen)
    leaves = [t.detach().clone().requires_grad_(True) for t in ins]

    def timed(fn):
        for _ in range(max(args.warmup, 1)):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(args.steps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        return round(statistics.median(ts), 3)

    def ours_fwd():
        with torch.no_grad():
            return ops.attention_span(*ins, g["metadata"], g["row_order"])

    def ours_fb(keep=True):
        out = ops.attention_span(*leaves, g["metadata"], g["row_order"], keep_logits=keep)
        return torch.autograd.grad(out, leaves, dout)

    clocks = ClockSampler(local)
    res = {"ours_fwd_ms": timed(ours_fwd), "ours_fwd_bwd_ms": timed(ours_fb),
           "ours_fwd_bwd_scores_recomputed_ms": timed(lambda: ours_fb(False))}
    mods, why = _load_reference_triton()
    if mods is None:
        res["reference"] = {"unavailable": why}
    else:
        md_ref = mods["triton_sparse_qk_autograd"].prepare_sparse_qk_edge_index_metadata(
            q_idx.to(torch.int32), n_idx.to(torch.int32), N, N2)
        qi32, ni32 = q_idx.to(torch.int32), n_idx.to(torch.int32)
        rleaves = [t.detach().clone().requires_grad_(True) for t in ins]

        def ref_fwd():
            with torch.no_grad():
                return reference_span(mods, *ins, qi32, ni32, md_ref, N)

        def ref_fb():
            out = reference_span(mods, *rleaves, qi32, ni32, md_ref, N)
            return torch.autograd.grad(out, rleaves, dout, allow_unused=True)

        try:
            o_ref = ref_fwd()
            o_us = ours_fwd()
            err = float((o_ref - o_us).abs().max()) / max(1.0, float(o_us.abs().max()))
            res["reference"] = {"fwd_ms": timed(ref_fwd), "fwd_bwd_ms": timed(ref_fb), "max_rel_diff_vs_ours": err}
            res["speedup_fwd"] = round(res["reference"]["fwd_ms"] / res["ours_fwd_ms"], 2)
            res["speedup_fwd_bwd"] = round(res["reference"]["fwd_bwd_ms"] / res["ours_fwd_bwd_ms"], 2)
            res["by_function"] = compare_kernel_functions(mods, ins, q_idx, n_idx, md_ref, g["metadata"], N, N2,
                                                          timed, dev)
        except Exception as exc:  # noqa: BLE001
            res["reference"] = {"unavailable": f"reference Triton kernels failed on this box: {exc!r}"[:300]}
    clk = clocks.stop()
    if rank == 0:
        line = {"metric": "attention span ms (forward; forward+backward)", "unit": "ms", "n_gpus": 1,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": False, "dtype": "f32",
                "data": "synthetic (seeded uniform box, seeded N(0,1) features)",
                "config": {"workload": f"attention span, uniform periodic box {N} atoms, ~{args.k} neighbours "
                                       f"within {CUTOFF} A", "edges": E, "expanded_nodes": N2, "heads": H,
                           "head_dim": D, "value_rows": C},
                "results": res, "gpu_launches": None, "clocks": clk}
        print(json.dumps(line))


# ------------------------------------------------------------------------------------------------
# The tensor-core projections alone: k_gemm_ws on the model's GEMM shapes
# ------------------------------------------------------------------------------------------------
GEMM_SHAPES = [  # (M, N, K, what) at the bench system: 97,865 atoms, 129,287 images, 3.13 M edges
    (97865 * 9, 1024, 256, "Q / K per-degree projections (pair product), all 9 irreps rows"),
    (97865, 512, 1536, "Q / K scalar MLP, first linear"),
    (97865, 1024, 512, "Q / K scalar MLP, second linear"),
    (97865 * 9, 256, 256, "proj_value / FFN per-degree linears"),
    (3131680, 128, 256, "edge radial MLP, first layer (radial basis x W)"),
    (3131680, 128, 128, "edge radial MLP, middle layer"),
    (3131680, 256, 128, "edge radial MLP, last layer (gate | inputhead)"),
]


def run_gemm(args, ws, rank, local):
    """Each of the model's GEMM shapes through ``linear.gemm`` (3xTF32 on tcgen05, fp32-accurate),
    CUDA events over ``--steps`` launches after ``--warmup``; TFLOP/s of fp32-accurate output (2MNK per
    product) against the 3xTF32 ceiling (a third of the dense tf32 rate, taken as half the measured
    bf16 rate) and against the measured bf16 peak."""
    from ubio_molfm_b200 import linear

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            bf16 = float(json.load(f)["bf16_tflops_sustained"])
    except Exception:
        bf16 = 1400.0   # the fallback sustained figure
    ceiling = bf16 / 2 / 3
    g = torch.Generator(device=dev).manual_seed(0)
    rows = []
    clocks = ClockSampler(local)
    for M, N, K, what in GEMM_SHAPES:
        a = torch.randn(M, K, device=dev, generator=g)
        b = torch.randn(N, K, device=dev, generator=g)
        bs = linear.split_tf32(b)
        out = torch.empty(M, N, device=dev)
        for _ in range(max(args.warmup, 1)):
            linear.gemm(a, b, out=out, b_split=bs)
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            linear.gemm(a, b, out=out, b_split=bs)
        t1.record()
        torch.cuda.synchronize()
        ms = t0.elapsed_time(t1) / args.steps
        tf = 2.0 * M * N * K / ms / 1e9
        rows.append({"M": M, "N": N, "K": K, "what": what, "ms": round(ms, 4), "tflops": round(tf, 1),
                     "frac_of_3xtf32_ceiling": round(tf / ceiling, 3), "frac_of_bf16_peak": round(tf / bf16, 3)})
        del a, b, bs, out
    # the two launch kinds the model runs most that the plain shapes above do not show: the Q / K pair
    # product per irreps row (epilogue P += o1 o2, projections kept for the backward) and the radial
    # basis formed inside the GEMM from the edge lengths
    N, C, Hd = 97865, 256, 512
    x = torch.randn(N, 9, C, device=dev, generator=g)
    w1 = torch.randn(3, Hd, C, device=dev, generator=g) / 16
    w2 = torch.randn(3, Hd, C, device=dev, generator=g) / 16
    bias = torch.zeros(1, 1, Hd, device=dev)
    lidx = [0, 1, 1, 1, 2, 2, 2, 2, 2]
    E, nb = 3131680, 256
    d = 6.0 * torch.rand(E, device=dev, generator=g)
    mu = torch.linspace(0, 6.0, nb, device=dev)
    coeff = -0.5 / (2.0 * (6.0 / (nb - 1))) ** 2
    wr = torch.randn(128, nb, device=dev, generator=g) / 16
    br = torch.zeros(128, device=dev)
    for what, fn, flop in [
            ("Q / K pair product, 9 irreps rows (9 launches, projections kept)",
             lambda: linear.so3_pair_product(x, w1, w2, bias, lidx, recompute=False), 2.0 * N * 9 * 2 * Hd * C),
            ("edge radial MLP first layer, basis formed on chip from 3.13 M edge lengths",
             lambda: linear.rbf_linear(d, mu, coeff, wr, br, on_chip=True), 2.0 * E * 128 * nb),
            ("edge radial MLP first layer, basis written by one kernel then the plain GEMM (the default)",
             lambda: linear.rbf_linear(d, mu, coeff, wr, br, on_chip=False), 2.0 * E * 128 * nb)]:
        for _ in range(max(args.warmup, 1)):
            fn()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            fn()
        t1.record()
        torch.cuda.synchronize()
        ms = t0.elapsed_time(t1) / args.steps
        tf = flop / ms / 1e9
        rows.append({"what": what, "ms": round(ms, 4), "tflops": round(tf, 1),
                     "frac_of_3xtf32_ceiling": round(tf / ceiling, 3), "frac_of_bf16_peak": round(tf / bf16, 3)})
    clk = clocks.stop()
    if rank == 0:
        print(json.dumps({"metric": "GEMM TFLOP/s of fp32-accurate output", "unit": "TFLOP/s", "n_gpus": 1,
                          "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "dtype": "f32",
                          "data": "synthetic N(0,1) operands", "ceiling_3xtf32_tflops": round(ceiling, 1),
                          "bf16_peak_tflops": bf16, "shapes": rows, "clocks": clk}))


# ------------------------------------------------------------------------------------------------
# Config 5's workload: NVE molecular dynamics through the MD API
# ------------------------------------------------------------------------------------------------
def run_md(args, ws, rank, local):
    """``--steps`` NVE velocity-Verlet steps at 0.5 fs (``TorchLangevin`` at zero friction with FixCom, on
    ``TorchAtoms`` with float64 state, forces from ``E2FormerCalculator``) on the bench system, from
    seeded Maxwell-Boltzmann velocities at 300 K.  Reports atom-steps/s of the MD loop and the drift of
    the total energy (potential + kinetic) over the run."""
    from ubio_molfm_b200 import _lib
    from ubio_molfm_b200.md import FS, E2FormerCalculator, TorchAtoms, TorchLangevin, maxwell_boltzmann
    from ubio_molfm_b200.synthetic import MASS, blob_in_water

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    model = make_model(dev)
    pos_np, Z_np, cell_np = blob_in_water(seed=100)
    masses = [MASS[int(z)] for z in Z_np]
    atoms = TorchAtoms(Z_np, pos_np, masses, cell_np, (True, True, True), device=dev)
    atoms.set_velocities(maxwell_boltzmann(masses, 300.0, torch.Generator().manual_seed(0), dev))
    atoms.calc = E2FormerCalculator(model, use_charge=False)
    dyn = TorchLangevin(atoms, 0.5 * FS, friction=0.0, fixcm=True)
    N = len(atoms)
    for _ in range(args.warmup):
        dyn.step()
    e0 = float(atoms.get_potential_energy() + atoms.get_kinetic_energy())
    ke0 = float(atoms.get_kinetic_energy())
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    launches0 = _lib.launch_count()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        dyn.step()
    t1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / args.steps
    e1 = float(atoms.get_potential_energy() + atoms.get_kinetic_energy())
    if rank == 0:
        print(json.dumps({
            "metric": "atom-steps/s (NVE MD, energy+forces per step)", "value": round(N * 1e3 / ms, 1),
            "unit": "atom-steps/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 3), "higher_is_better": True, "dtype": "f32 model, f64 integrator state",
            "data": "synthetic (seeded blob-in-water periodic system, seeded random weights, MB velocities 300 K)",
            "config": {"workload": "NVE velocity Verlet, 0.5 fs, FixCom, on the 97,865-atom bench system",
                       "atoms": N, "dt_fs": 0.5},
            "energy_drift": {"total_energy_start_eV": e0, "total_energy_end_eV": e1,
                             "drift_eV": e1 - e0, "drift_per_atom_eV": (e1 - e0) / N,
                             "drift_over_initial_kinetic": (e1 - e0) / ke0},
            "gpu_launches": _lib.launch_count() - launches0, "clocks": clk}))


def main():
    args = parse()
    ws, rank, local = dist_init(args)
    if args.workload == "molecules":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the molecules workload has no CPU reference "
                                                                  "arm; use the default workload"}))
        else:
            run_molecules(args, ws, rank, local)
    elif args.workload == "span":
        run_span(args, ws, rank, local)
    elif args.workload == "gemm":
        run_gemm(args, ws, rank, local)
    elif args.workload == "md":
        run_md(args, ws, rank, local)
    elif args.workload == "model":
        if args.impl == "reference":
            run_reference_model(args, ws, rank)
        else:
            run_model(args, ws, rank, local)
    elif args.impl == "reference":
        run_reference(args, ws, rank)
    else:
        run_ours(args, ws, rank, local)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
