"""Torch restatement of the reference's auxiliary losses -- TEST INFRASTRUCTURE ONLY.

The checker of the fused router-head / aux-loss kernels: the reference's own
torch expressions for router_z_loss, load_balance_loss (with its expert size
groups) and compute_loss, evaluated with autograd so that the tests can also
compare gradients.  Nothing in the product imports it.

Follows triton_moe/moe.py:108-146 (size groups and their buffers),
:253-272 (the three losses and f_i) and :276-303 (_compute_load_balance_loss).
"""

from __future__ import annotations

import torch


def _groups(expert_sizes):
    """(expert -> group id or -1, group sizes): size classes with more than one
    expert form a load-balance group; singleton classes are left out
    (moe.py:108-146)."""
    expert_to_group, group_sizes = [], []
    for count, _size in expert_sizes:
        expert_to_group += [len(group_sizes) if count > 1 else -1] * count
        if count > 1:
            group_sizes.append(count)
    return expert_to_group, group_sizes


def load_balance_loss(expert_sizes, router_probs: torch.Tensor, f_i: torch.Tensor) -> torch.Tensor:
    """moe.py:276-303: uniform widths -> E * f.p; no group -> f.p; else the mean
    over groups of group_size * sum_{e in group} f_e p_e."""
    widths = [w for c, w in expert_sizes for _ in range(c)]
    E = len(widths)
    p_i = router_probs.mean(dim=0)
    if len(set(widths)) == 1:
        return E * (f_i.float() @ p_i.float())
    e2g, sizes = _groups(expert_sizes)
    if not sizes:
        return f_i.float() @ p_i.float()
    fi_pi = f_i.float() * p_i.float()
    membership = torch.zeros(E, len(sizes), dtype=fi_pi.dtype, device=fi_pi.device)
    for e, g in enumerate(e2g):
        if g >= 0:
            membership[e, g] = 1.0
    valid = torch.tensor([e for e, g in enumerate(e2g) if g >= 0], device=fi_pi.device)
    group_sums = fi_pi.index_select(0, valid) @ membership.index_select(0, valid)
    return (torch.tensor(sizes, dtype=fi_pi.dtype, device=fi_pi.device) * group_sums).mean()


def aux_losses(expert_sizes, router_logits, router_probs, tokens_per_expert, dtype):
    """moe.py:253-272: ({router_z_loss, load_balance_loss, compute_loss}, f_i)."""
    widths = [w for c, w in expert_sizes for _ in range(c)]
    mean_w = sum(widths) / len(widths)
    wn = torch.tensor([w / mean_w for w in widths], dtype=torch.float32,
                      device=router_logits.device)
    router_z_loss = torch.logsumexp(router_logits, dim=-1).pow(2).mean()
    f_i = (tokens_per_expert.float() / tokens_per_expert.sum()).to(dtype)
    lb = load_balance_loss(expert_sizes, router_probs, f_i)
    compute_loss = (router_probs @ wn.to(router_probs.dtype)).mean()
    return {"router_z_loss": router_z_loss, "load_balance_loss": lb,
            "compute_loss": compute_loss}, f_i
