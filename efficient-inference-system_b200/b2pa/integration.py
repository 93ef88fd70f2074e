"""Installs this backend into a checkout of the reference serving stack.

The reference calls its attention backend from exactly one place,
``CausalSelfAttention.forward`` (src/model/attention.py:56-62):
``kv_cache.append_batch(...)`` followed by ``paged_attention(...)``.  Because
``src/model/attention.py:6`` binds ``paged_attention`` by name, both that
module's global and ``src.kernels.paged_attention.paged_attention`` are
rebound here; ``BatchedPagedKVCache.append_batch`` is replaced on the class.

After ``install_into_reference()``, a model built with the reference's
default ``attention_backend="triton_paged"`` runs its paged attention and KV
scatter on the b2pa kernels, with the reference's own pools, block tables and
schedulers.  ``"paged_reference"`` and CPU tensors keep the reference's torch
path.  The returned handle's ``uninstall()`` restores the originals.
"""
from __future__ import annotations

import importlib
from dataclasses import dataclass


@dataclass
class InstallHandle:
    originals: dict
    fused_before: bool = False

    def uninstall(self) -> None:
        from .paged_kv import set_fused_append

        for (module, attr), value in self.originals.items():
            setattr(module, attr, value)
        set_fused_append(self.fused_before)


def install_into_reference(package: str = "src", fuse_append: bool = False) -> InstallHandle:
    """Routes the reference's GPU attention backend through b2pa.

    ``package`` is the import name of the reference's source package (the
    reference's repository root must be on ``sys.path``).  With
    ``fuse_append`` a decode step's append_batch leaves its K/V row copy to
    the paged_attention call that follows it, which performs it in its own
    launch (``b2pa.set_fused_append``); the reference's forward always makes
    that pair of calls back to back.
    """
    from .attention import paged_attention as b2pa_paged_attention
    from .paged_kv import append_batch_into, set_fused_append

    kernels_mod = importlib.import_module(f"{package}.kernels.paged_attention")
    model_attn_mod = importlib.import_module(f"{package}.model.attention")
    cache_mod = importlib.import_module(f"{package}.cache.paged_kv")
    kernels_pkg = importlib.import_module(f"{package}.kernels")

    orig_pa = kernels_mod.paged_attention
    orig_append = cache_mod.BatchedPagedKVCache.append_batch

    def paged_attention(backend, q, kv_cache, current_lengths):
        if backend == "paged_reference" or not q.is_cuda:
            return orig_pa(backend=backend, q=q, kv_cache=kv_cache, current_lengths=current_lengths)
        if backend != "triton_paged":
            raise ValueError(f"Unsupported paged attention backend: {backend}")
        return b2pa_paged_attention("b200_paged", q, kv_cache, current_lengths)

    def append_batch(self, k_new, v_new, current_lengths=None):
        if not k_new.is_cuda:
            return orig_append(self, k_new, v_new, current_lengths)
        return append_batch_into(self, k_new, v_new, current_lengths)

    originals = {
        (kernels_mod, "paged_attention"): orig_pa,
        (model_attn_mod, "paged_attention"): model_attn_mod.paged_attention,
        (kernels_pkg, "paged_attention"): getattr(kernels_pkg, "paged_attention", orig_pa),
        (cache_mod.BatchedPagedKVCache, "append_batch"): orig_append,
    }
    kernels_mod.paged_attention = paged_attention
    model_attn_mod.paged_attention = paged_attention
    kernels_pkg.paged_attention = paged_attention
    cache_mod.BatchedPagedKVCache.append_batch = append_batch
    return InstallHandle(originals, set_fused_append(fuse_append))
