"""Golden of the FL2AV hook's ``sol_attn`` backend (F/streaming/attention_hook.py:909-991,
1361-1492), run on CPU by ``make_golden.py hook_sol.npz`` in a process of its own (Triton's
CPU interpreter must be chosen before Triton is imported).

Three clean commits (dense in the commit modes), then a NOISY call at denoise step 1 through
all layers; layer 0 (a dense layer) and layer 2 (routed) outputs are kept, for the default
policy and for ``sol_attn_route_current_video``. The interpreter mishandles bf16 buffers, so
the adapter's own buffers are float32 during its call (``torch.bfloat16`` stands for float32
there) and its inputs are the hook's bf16 rows as float32; the hook itself runs in bf16 on CPU
tensors that report ``is_cuda``.

    python tests/golden/make_hook_sol.py OUT.npz
"""

from __future__ import annotations

import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402

import make_golden  # noqa: E402
from inputs import sol_hook_inputs  # noqa: E402


def main(path: str) -> None:
    make_golden._import_reference()
    import torch
    import digitalhuman_h3.inference.sol_attention as sol
    import digitalhuman_h3.streaming.attention_hook as fhook
    import digitalhuman_h3.streaming.cache as fcache

    fcache._validate_av_pair = lambda pair, contract, *, layer: None
    fcache._validate_video_pair = lambda pair, contract, *, layer: None
    rectangular = sol.sol_attn_rectangular

    def float32_adapter(query, key, value, **kw):
        q, k, v = (torch.Tensor(t).float() for t in (query, key, value))
        saved, torch.bfloat16 = torch.bfloat16, torch.float32
        try:
            out = rectangular(q, k, v, **kw)
        finally:
            torch.bfloat16 = saved
        return out.to(torch.bfloat16)

    sol.sol_attn_rectangular = float32_adapter

    class CudaFlagged(torch.Tensor):
        @property
        def is_cuda(self):
            return True

    def t(x: np.ndarray, dtype=torch.bfloat16):
        return torch.from_numpy(np.ascontiguousarray(x)).to(dtype).as_subclass(CudaFlagged)

    class Attn:
        softmax_scale = 128 ** -0.5

    history, y = sol_hook_inputs()
    arrays: dict[str, np.ndarray] = {}
    for name, route_video in (("default", False), ("route_video", True)):
        contract = fcache.KVContract(local_heads=2, head_dim=128)
        cache = fcache.CleanAVKVCache(contract)
        hook = fhook.H3StreamingAttentionHook(cache, attention_backend="sol_attn", sol_attn_tau=0.5,
                                              sol_attn_route_current_video=route_video)
        for step, x in enumerate(history + [y]):
            noisy = step == len(history)
            mode = fhook.HookMode.NOISY if noisy else fhook.HookMode.CLEAN_COMMIT
            if not noisy:
                cache.begin_clean_commit(cache.committed_blocks)
            hook.activate(mode=mode, block_index=cache.committed_blocks, full_prefix=None,
                          **({"denoise_step_index": 1} if noisy else {}))
            for layer in contract.layer_names:
                out = hook(attention=Attn(), layer_name=layer, query=t(x["q"]), key=t(x["k"]),
                           value=t(x["v"]), token_tags=t(x["token_tags"], torch.int64),
                           commit_mask=t(x["commit_mask"], torch.bool), cu_seqlens=None,
                           cu_seqlens_host=tuple(x["cu_seqlens"]), max_seqlen=320)
                if noisy and layer in ("blocks.0.attn", "blocks.2.attn"):
                    o = torch.Tensor(out).float().numpy()
                    arrays[f"{name}_{layer.split('.')[1]}"] = (o.view(np.uint32) >> 16).astype(
                        np.uint16)  # bf16 bits
            hook.deactivate()
            if not noisy:
                cache.commit()
        receipt = hook.sol_attn_receipt()
        arrays[f"{name}_calls"] = np.array([receipt["kernel_calls"], receipt["dense_calls"]])
    np.savez_compressed(path, **arrays)


if __name__ == "__main__":
    main(sys.argv[1])
