"""Seeded synthetic workloads for the benchmark configurations.

Shapes and value distributions follow the reference's benchmark configs
(random-init Qwen3-Next sparse-MoE block: H=2048, I=512, E=512, top-10, MLX
4-bit affine experts with group 64, nibbles uniform in 0..15, bf16 scales
U(0.002, 0.02) and biases -8*scale; router and shared-gate weights N(0,
0.02); inputs N(0, 1)). Dense tensors come from numpy ``PCG64(seed)``; expert
weights are filled on the device by a counter hash of (seed, layer, expert)
so that a 16 GB pool is generated in well under a second and any expert can
be regenerated on its own.
"""
from __future__ import annotations

import numpy as np
import torch

from .moe_block import MoeBlock, Workspace
from .pool import QuantPool, expert_seed, make_table

H, I, E, K = 2048, 512, 512, 10
SHARED_ID = 100_000  # expert-seed id of a layer's shared expert


def normal_bf16(rng: np.random.Generator, shape, std: float, device) -> torch.Tensor:
    a = rng.standard_normal(shape, dtype=np.float32) * np.float32(std)
    return torch.from_numpy(a).to(torch.bfloat16).to(device)


def make_layer(seed: int, layer: int, pool: QuantPool, experts_in_slots, device="cuda",
               hidden=H, inter=I, num_experts=E, top_k=K, router_bias=None,
               workspace: Workspace | None = None, bias_mul: float = -8.0) -> MoeBlock:
    """One synthetic MoE layer whose ``pool`` slot ``s`` holds expert
    ``experts_in_slots[s]`` (filled here)."""
    rng = np.random.Generator(np.random.PCG64([seed, layer]))
    wr = normal_bf16(rng, (num_experts, hidden), 0.02, device)
    wsg = normal_bf16(rng, (hidden,), 0.02, device)
    experts = [int(e) for e in experts_in_slots]
    pool.fill_synthetic_many(range(len(experts)), [expert_seed(seed, layer, e) for e in experts],
                             bias_mul=bias_mul)
    shared = QuantPool.empty_blob(1, hidden, inter, pool.bits, pool.group, device)
    shared.fill_synthetic_many([0], [expert_seed(seed, layer, SHARED_ID)], bias_mul=bias_mul)
    table = make_table(num_experts, {int(e): s for s, e in enumerate(experts_in_slots)}, device)
    return MoeBlock(wr, table, pool, shared, wsg, top_k=top_k, router_bias=router_bias,
                    workspace=workspace)


def input_tokens(seed: int, T: int, hidden=H, device="cuda") -> torch.Tensor:
    rng = np.random.Generator(np.random.PCG64([seed, 999_999]))
    return normal_bf16(rng, (T, hidden), 1.0, device)


def config0(seed: int = 0, device="cuda", hidden=H, inter=I, num_experts=E, top_k=K):
    """Config 0: one sparse-MoE block, all experts resident (identity table),
    decode T=1."""
    pool = QuantPool.empty_blob(num_experts, hidden, inter, 4, 64, device)
    blk = make_layer(seed, 0, pool, range(num_experts), device, hidden, inter,
                     num_experts, top_k)
    x = input_tokens(seed, 1, hidden, device)
    return blk, x


def zipf_bias(seed: int, num_experts: int = E, s: float = 1.1) -> np.ndarray:
    """Router logit bias ``b_e = ln Zipf_pmf(rank(e); s)`` with the rank of
    each expert from a seeded permutation (config 2's skewed routing)."""
    rng = np.random.Generator(np.random.PCG64([seed, 424242]))
    ranks = rng.permutation(num_experts) + 1
    pmf = ranks.astype(np.float64) ** -s
    pmf /= (np.arange(1, num_experts + 1, dtype=np.float64) ** -s).sum()
    return np.log(pmf).astype(np.float32)


def config2(seed: int = 2, T: int = 32768, device="cuda", hidden=H, inter=I, num_experts=E,
            top_k=K):
    """Config 2: one sparse-MoE layer for expert-major prefill of T tokens;
    all experts resident (identity table), Zipf(1.1) router bias."""
    pool = QuantPool.empty_blob(num_experts, hidden, inter, 4, 64, device)
    bias = torch.from_numpy(zipf_bias(seed, num_experts)).to(device)
    blk = make_layer(seed, 0, pool, range(num_experts), device, hidden, inter, num_experts,
                     top_k, router_bias=bias)
    x = input_tokens(seed, T, hidden, device)
    return blk, x


def fresh_input_seed(seed: int, layer: int) -> int:
    """Seed of the fresh per-layer input of :class:`DecodeStack` (``fresh``)."""
    return seed * 1000 + layer + 1


class DecodeStack:
    """Config 1: ``L`` stacked MoE blocks, T tokens (MTP K=3 verify uses 4).

    Layer ``l``'s experts resolve through its own slot table into rows
    ``[l*cap, (l+1)*cap)`` of one packed HBM pool. Each block computes
    ``out <- x + MoE_l(rmsnorm(x))`` (the decoder's pre-norm residual around
    the MoE). With ``fresh=False`` the layers form a chain (``x_{l+1}`` is
    layer ``l``'s output); with random-init weights that chain drifts
    towards a common direction and routes fewer distinct experts per layer
    than real hidden states do. With ``fresh=True`` every layer gets its own
    seeded N(0, 1) input (the launches still follow one another on the
    stream), so the routes of different layers are independent, as they are
    for real hidden states: about 39 distinct experts per layer at T=4.
    """

    def __init__(self, seed: int = 1, layers: int = 48, cap: int = 192, T: int = 4,
                 device="cuda", hidden=H, inter=I, num_experts=E, top_k=K,
                 norm_eps: float = 1e-6, fresh: bool = False):
        self.seed, self.L, self.cap, self.T = seed, layers, cap, T
        self.fresh = fresh
        self.hidden, self.inter, self.num_experts, self.top_k = hidden, inter, num_experts, top_k
        self.norm_eps = norm_eps
        self.device = device
        self.big = QuantPool.empty_blob(layers * cap, hidden, inter, 4, 64, device)
        self.ws = Workspace(device)
        self.blocks: list[MoeBlock] = []
        self.slot_experts: list[list[int]] = []
        for l in range(layers):
            rng = np.random.Generator(np.random.PCG64([seed, l, 7]))
            perm = rng.permutation(num_experts)[:cap].tolist()
            self.slot_experts.append(perm)
            blk = make_layer(seed, l, self.big.view(l * cap, cap), perm, device, hidden,
                             inter, num_experts, top_k, workspace=self.ws)
            self.blocks.append(blk)
        self.x = input_tokens(seed, T, hidden, device)
        self.hs = [torch.empty((T, hidden), dtype=torch.bfloat16, device=device)
                   for _ in range(layers + 1)]
        self.hs[0].copy_(self.x)
        # fresh inputs: one [L, T, H] tensor (one host->device copy per step)
        self.xs = (torch.stack([input_tokens(fresh_input_seed(seed, l), T, hidden, device)
                                for l in range(layers)]) if fresh else None)

    def layer_input(self, l: int) -> torch.Tensor:
        """The input (and residual) of layer ``l``."""
        return self.xs[l] if self.fresh else self.hs[l]

    def ensure_resident(self, max_rounds: int = 4) -> int:
        """Make every expert routed by the stack's fixed input resident.

        Routes are drawn first (one pass layer by layer); a routed expert that
        is not in the table replaces a slot whose expert is not routed, then the
        layer is recomputed. Returns the number of replacements."""
        swaps = 0
        for l, blk in enumerate(self.blocks):
            for _ in range(max_rounds):
                dbg = blk.new_debug(self.T, self.device)
                xin = self.layer_input(l)
                blk.decode(xin, out=self.hs[l + 1], residual=xin, debug=dbg,
                           norm_eps=self.norm_eps)
                routed = set(dbg["inds"].flatten().tolist())
                slots = self.slot_experts[l]
                missing = [e for e in routed if e not in slots]
                if not missing:
                    break
                free = [s for s, e in enumerate(slots) if e not in routed]
                for e, s in zip(missing, free):
                    slots[s] = e
                    swaps += 1
                placed = list(zip(missing, free))
                blk.pool.fill_synthetic_many([s for _, s in placed],
                                             [expert_seed(self.seed, l, e) for e, _ in placed])
                blk.slot_table.copy_(make_table(self.num_experts,
                                                {e: s for s, e in enumerate(slots)},
                                                self.device))
        torch.cuda.synchronize()
        return swaps

    def step(self, stream=None, trace=None):
        """One whole-stack step: 48 chained MoE blocks over the T tokens.
        ``trace`` (int64 [L, 16] device tensor) records per-layer kernel spans and markers."""
        for l, blk in enumerate(self.blocks):
            xin = self.layer_input(l)
            blk.decode(xin, out=self.hs[l + 1], residual=xin,
                       norm_eps=self.norm_eps, stream=stream,
                       trace=None if trace is None else trace[l])
        return self.hs[-1]

    def token_routes(self, t: int) -> list[list[int]]:
        """Routed experts of token ``t`` per layer for the fixed input (tokens
        are routed independently, so a single-token chain of token ``t``
        sees the same experts)."""
        out = []
        for l, blk in enumerate(self.blocks):
            dbg = blk.new_debug(self.T, self.device)
            xin = self.layer_input(l)
            blk.decode(xin, out=torch.empty_like(xin), residual=xin,
                       debug=dbg, norm_eps=self.norm_eps)
            out.append(dbg["inds"][t].tolist())
        return out

    def unique_experts(self) -> list[int]:
        """Distinct routed experts per layer for the fixed input (U_l)."""
        out = []
        for l, blk in enumerate(self.blocks):
            dbg = blk.new_debug(self.T, self.device)
            xin = self.layer_input(l)
            blk.decode(xin, out=torch.empty_like(xin), residual=xin,
                       debug=dbg, norm_eps=self.norm_eps)
            out.append(len(set(dbg["inds"].flatten().tolist())))
        return out


def layer_to_host(blk: MoeBlock, experts) -> dict:
    """Copy a block's router, shared expert and the pool slots of ``experts``
    to host numpy (uint32 words, uint16 bf16 bits, float32 dense weights).

    The returned pool is compact: ``table[e]`` indexes it for the copied
    experts and is -1 for every other expert."""
    import numpy as np
    from .pool import KEYS
    full_table = blk.slot_table.cpu().numpy()
    experts = sorted({int(e) for e in experts if full_table[int(e)] >= 0})
    parts = [blk.pool.to_numpy_slot(int(full_table[e])) for e in experts]
    pool = {k: np.concatenate([p[k] for p in parts]) for k in KEYS} if parts else None
    table = np.full_like(full_table, -1)
    for i, e in enumerate(experts):
        table[e] = i
    return {"wr": blk.router_w.float().cpu().numpy(),
            "wsg": blk.shared_gate_w.float().cpu().numpy(),
            "table": table, "pool": pool, "shared": blk.shared.to_numpy_slot(0),
            "hidden": blk.hidden, "inter": blk.inter, "group": blk.pool.group,
            "bits": blk.pool.bits,
            "logit_bias": None if blk.router_bias is None else blk.router_bias.cpu().numpy()}
