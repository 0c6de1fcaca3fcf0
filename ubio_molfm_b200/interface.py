"""The reference's model-interface boundary over :class:`~ubio_molfm_b200.model.E2FormerPotential`.

* :func:`collate_systems` -- ``dict_to_model_input`` / ``collate_fn`` (interface/data_utils.py:37-80,
  data/collator.py:25-52) without ASE: per-structure dicts (``atoms``, ``coords``, ``charge``,
  ``multiplicity``, ``cell``, ``pbc``) -> the padded batch the model takes (``pos [B,L,3]``,
  ``atomic_numbers [B,L]``, ``atom_masks [B,L]``, ``charge [B,1]``, ``multiplicity [B,1]``,
  ``cell [B,3,3]``, ``pbc [B,3]``, ``num_atoms [B,1]``, ``data_name``).
* :class:`E2FormerModelInterface` -- ``predict(model_input, need_force)`` of
  interface/model_interface.py:64-281: takes that batch and returns ``pred_energy [B]``,
  ``pred_forces [B,L,3]`` (zero on padding) and ``pred_energy_per_atom [B]``, the keys of
  ``MDEnergyForceMultiHead.forward`` (pipeline/head.py:552-580).  ``use_tf32`` selects the single-pass
  TF32 projection mode (the reference's ``configure_tf32``, tasks/pretrain_smallmol.py:212-226).

Periodic systems are evaluated one per model call; non-periodic systems of a batch are evaluated
together (systems do not see each other).
"""
from __future__ import annotations

import contextlib

import numpy as np
import torch

from . import linear
from .model import E2FormerPotential

# keys of the reference backbone config that the potential takes (config_file/backbone_config/e2former.yaml)
_BACKBONE_KEYS = ("irreps_node_embedding", "num_layers", "max_neighbors", "max_radius", "basis_type",
                  "number_of_basis", "num_attn_heads", "attn_scalar_head", "irreps_head", "norm_layer", "alpha_drop",
                  "tp_type", "attn_type", "atom_type_cnt", "edge_embedtype", "ffn_type", "avg_degree", "with_cluster",
                  "encoder", "encoder_embed_dim", "pbc_expanded_num_cell_per_direction")


def collate_systems(systems, data_name="default", device="cpu", pos_dtype=torch.float32):
    """interface/data_utils.py:37-80 + data/collator.py:25-52 on plain dicts."""
    n_max = max(len(s["atoms"]) for s in systems)
    B = len(systems)
    pos = torch.zeros((B, n_max, 3), dtype=pos_dtype)
    Z = torch.zeros((B, n_max), dtype=torch.int32)
    mask = torch.zeros((B, n_max), dtype=torch.bool)
    cell = torch.zeros((B, 3, 3), dtype=torch.float32)
    pbc = torch.zeros((B, 3), dtype=torch.int32)
    charge = torch.zeros((B, 1), dtype=torch.int32)
    mult = torch.ones((B, 1), dtype=torch.int32)
    num = torch.zeros((B, 1), dtype=torch.int32)
    for b, s in enumerate(systems):
        n = len(s["atoms"])
        pos[b, :n] = torch.as_tensor(np.asarray(s["coords"]), dtype=pos_dtype).reshape(-1, 3)
        Z[b, :n] = torch.as_tensor(np.asarray(s["atoms"]), dtype=torch.int32)
        mask[b, :n] = True
        if s.get("cell") is not None:
            cell[b] = torch.as_tensor(np.asarray(s["cell"]), dtype=torch.float32)
        if s.get("pbc") is not None:
            pbc[b] = torch.as_tensor(np.asarray(s["pbc"]).astype(np.int32))
        charge[b, 0] = int(s.get("charge", 0))
        mult[b, 0] = int(s.get("multiplicity", 1))
        num[b, 0] = n
    out = {"pos": pos, "atomic_numbers": Z, "atom_masks": mask, "cell": cell, "pbc": pbc, "charge": charge,
           "multiplicity": mult, "num_atoms": num}
    out = {k: v.to(device) for k, v in out.items()}
    out["data_name"] = [data_name]
    return out


@contextlib.contextmanager
def projection_precision(mode):
    """``"fp32"`` (3xTF32 GEMMs, the parity mode) or ``"tf32"`` (single-pass TF32 GEMMs) for the
    projections run inside the block."""
    if mode not in ("fp32", "tf32"):
        raise ValueError(f"projection precision {mode!r}: expected 'fp32' or 'tf32'")
    old = linear.PASSES
    linear.PASSES = 1 if mode == "tf32" else 3
    try:
        yield
    finally:
        linear.PASSES = old


class E2FormerModelInterface:
    """interface/model_interface.py:64-281 over a B200 potential.

    Either pass a built ``model`` (an :class:`E2FormerPotential`), or a ``backbone_config`` dict (the
    keys of config_file/backbone_config/e2former.yaml; a yaml path is read with ``yaml``) to build one
    with random weights, optionally loaded from ``checkpoint_path`` (a reference ``MolfmAtomic``
    checkpoint: ``torch.load(...)["model"]``, ``head.energy_heads.<head_name>``)."""

    def __init__(self, model=None, backbone_config=None, checkpoint_path=None, head_name=None, device="cuda:0",
                 use_tf32=False, use_faiss=True, use_compile=False, ref_energy=None, memory_saving="auto"):
        if use_compile:
            raise NotImplementedError("use_compile: this build runs its own CUDA kernels, not torch.compile")
        self.device = torch.device(device)
        self.use_tf32, self.use_faiss, self.head_name = use_tf32, use_faiss, head_name
        if model is None:
            if backbone_config is None:
                raise ValueError("pass a model or a backbone_config")
            if isinstance(backbone_config, str):
                import yaml

                with open(backbone_config, "r", encoding="utf-8") as f:
                    backbone_config = yaml.safe_load(f)
            cfg = {k: v for k, v in backbone_config.items() if k in _BACKBONE_KEYS}
            model = E2FormerPotential(memory_saving=memory_saving, use_faiss=use_faiss, **cfg)
            if checkpoint_path not in (None, "none"):
                sd = torch.load(checkpoint_path, map_location="cpu")
                model.load_reference_state_dict(sd.get("model", sd), head_name=head_name, strict=False)
        self.model = model.to(self.device).eval()
        self.ref_energy = None if ref_energy is None else torch.as_tensor(ref_energy, device=self.device)

    def predict(self, model_input, need_force=True):
        """``model_input``: the collated batch (:func:`collate_systems`); returns a dict with
        ``pred_energy [B]``, ``pred_forces [B,L,3]``, ``pred_energy_per_atom [B]``."""
        pos = model_input["pos"]
        mask = model_input["atom_masks"].to(pos.device).bool()
        B, L = mask.shape
        dev = self.device
        Z = model_input["atomic_numbers"].to(dev).reshape(B, L).long()
        pbc = torch.as_tensor(model_input.get("pbc", torch.zeros(B, 3))).reshape(B, 3).bool()
        cell = torch.as_tensor(model_input.get("cell", torch.zeros(B, 3, 3))).reshape(B, 3, 3).float().cpu()
        charge = model_input.get("charge")
        mult = model_input.get("multiplicity")
        if charge is not None:
            charge = torch.as_tensor(charge).reshape(B)
            mult = torch.ones_like(charge) if mult is None else torch.as_tensor(mult).reshape(B)
        energy = torch.zeros(B, device=dev, dtype=torch.float32)
        forces = torch.zeros((B, L, 3), device=dev, dtype=torch.float32)
        counts = mask.sum(-1).cpu()
        periodic = pbc.any(-1).cpu()
        with projection_precision("tf32" if self.use_tf32 else "fp32"):
            for b in torch.nonzero(periodic).flatten().tolist():
                n = int(counts[b])
                e, f = self.model(pos[b, :n].to(dev), Z[b, :n], cell[b], [bool(v) for v in pbc[b].tolist()],
                                  None, need_force,
                                  None if charge is None else charge[b:b + 1], None if mult is None else mult[b:b + 1])
                energy[b] = e.reshape(-1)[0]
                if need_force:
                    forces[b, :n] = f
            mol = torch.nonzero(~periodic).flatten()
            if mol.numel():
                m = mask[mol].to(dev)
                sel_pos = pos[mol].to(dev)[m]
                sel_Z = Z[mol][m]
                batch = torch.arange(mol.numel(), device=dev).unsqueeze(1).expand(-1, L)[m]
                e, f = self.model(sel_pos, sel_Z, None, (False, False, False), batch, need_force,
                                  None if charge is None else charge[mol], None if mult is None else mult[mol])
                energy[mol.to(dev)] = e.reshape(-1)
                if need_force:
                    fb = forces[mol.to(dev)]
                    fb[m] = f
                    forces[mol.to(dev)] = fb
        if self.ref_energy is not None:
            energy = energy + (self.ref_energy[Z] * mask.to(dev)).sum(-1)
        out = {"pred_energy": energy, "pred_energy_per_atom": energy / counts.to(dev).clamp(min=1)}
        if need_force:
            out["pred_forces"] = forces
        return out

    def __call__(self, *args, **kwargs):
        return self.predict(*args, **kwargs)
