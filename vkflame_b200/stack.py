"""A GGUF-driven decoder linear stack on the per-token chain kernel.

Loads the linear weights of a llama-family decoder (tensor names
``blk.<i>.attn_q.weight`` ... ``output.weight``; architectures llama and
qwen2 and any other that uses these names) from a GGUF file, shards them by
output rows over the ranks, and runs one decode step as one persistent
kernel (``vkflame_chain_run``).  Per layer: q and k fused into one link
(same input and format: their rows concatenated), v, o, gate and up fused,
down; then the output head.  Data flow, as in the stack benchmark: q/k and v
read the layer input (the previous layer's down output; the token's input
row for layer 0), o reads q/k's output (standing in for attention), gate/up
reads o's, down reads gate/up's, the head reads the last down's.  The
norms, rotary embedding, attention and the SwiGLU product between the
linears are not part of this stack.

Formats: Q4_K, Q5_K and Q6_K (the Q4_K_M family); another format raises.
"""
from __future__ import annotations

import warnings

import numpy as np

from . import gguf, rt, shard


def _layer_names(i: int) -> dict:
    b = f"blk.{i}."
    return {"q": b + "attn_q.weight", "k": b + "attn_k.weight", "v": b + "attn_v.weight",
            "o": b + "attn_output.weight", "gate": b + "ffn_gate.weight", "up": b + "ffn_up.weight",
            "down": b + "ffn_down.weight"}


def plan(g: gguf.GGUFFile) -> list:
    """The stack's links: (name, format, K, N, [tensor names whose rows are
    concatenated], input link name or None)."""
    arch = g.metadata.get("general.architecture", "llama")
    layers = int(g.metadata.get(f"{arch}.block_count", 0))
    if layers <= 0:
        raise ValueError("GGUF metadata has no block_count")
    links = []

    def link(name, tensors, src):
        kinds = set()
        K = None
        N = 0
        for t in tensors:
            kind, k, n, _ = g.weight(t)
            kinds.add(kind)
            if K is not None and k != K:
                raise ValueError(f"{name}: fused tensors with different K")
            K, N = k, N + n
        if len(kinds) != 1:
            # different formats cannot share a link: split
            return [link(f"{name}.{j}", [t], src)[0] for j, t in enumerate(tensors)]
        kind = kinds.pop()
        if kind not in (rt.Q4_K, rt.Q5_K, rt.Q6_K):
            raise ValueError(f"{name}: format {kind} not supported by the chain kernel (Q4_K, Q5_K, Q6_K)")
        return [(name, kind, K, N, list(tensors), src)]

    prev = None
    for i in range(layers):
        n = _layer_names(i)
        qk = link(f"{i}.qk", [n["q"], n["k"]], prev)
        links += qk
        links += link(f"{i}.v", [n["v"]], prev)
        links += link(f"{i}.o", [n["o"]], qk[0][0])
        gu = link(f"{i}.gate_up", [n["gate"], n["up"]], f"{i}.o")
        links += gu
        links += link(f"{i}.down", [n["down"]], gu[0][0])
        prev = f"{i}.down"
    links += link("head", ["output.weight" if "output.weight" in g.tensors else "token_embd.weight"], prev)
    return links


class GGUFStack:
    """One rank's shard of a GGUF model's linear stack, ready to run.

    world / rank / dist: column sharding over ranks (one process per GPU,
    torch.distributed for the handle exchange only); world 1 runs alone."""

    def __init__(self, path, world: int = 1, rank: int = 0, dist=None, stream: int = 0):
        import torch
        from .gather import GatherGroup
        self.file = gguf.read(path)
        self.links = plan(self.file)
        self.world, self.rank, self.stream = world, rank, stream
        self.gg = GatherGroup(dist, world, rank)
        K0 = self.links[0][2]
        self.x = torch.zeros((1, K0), dtype=torch.float16, device="cuda")
        self.weights, self.outs, cl = [], {}, []
        self.weight_bytes = 0
        index = {}
        for name, kind, K, N, tensors, src in self.links:
            rows = np.concatenate([self.file.weight(t)[3] for t in tensors]) if len(tensors) > 1 else \
                self.file.weight(tensors[0])[3]
            r0, r1 = shard.row_range(N, world, rank)
            with warnings.catch_warnings():
                # a read-only view of the mapped file, only read (copied to the device)
                warnings.simplefilter("ignore", UserWarning)
                w = torch.from_numpy(np.ascontiguousarray(rows[r0:r1]).reshape(-1)).cuda()
            self.weights.append(w)
            self.weight_bytes += w.numel()
            out = self.gg.buffer(N)
            self.outs[name] = out
            if src is not None and src not in index:
                raise ValueError(f"{name}: input link {src} not found")
            cl.append(self.gg.chain_linear(w.data_ptr(), kind, K, r1 - r0, out,
                                           x_src=index[src] if src is not None else -1,
                                           x_plain=self.x.data_ptr() if src is None else 0))
            index[name] = len(cl) - 1
        self.chain = rt.Chain(cl, world, rank)
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()

    def step(self, x=None) -> None:
        """One decode step (asynchronous on `stream`); x: the token's input
        row (hidden values), copied in first when given."""
        import torch
        if x is not None:
            row = torch.as_tensor(np.asarray(x, np.float16).reshape(1, -1))
            # the copy goes on the chain's own stream, so the kernel reads it
            # after it lands whatever stream torch has current
            s = torch.cuda.ExternalStream(self.stream) if self.stream else torch.cuda.default_stream()
            with torch.cuda.stream(s):
                self.x.copy_(row)
        self.chain.run(self.stream)

    def output(self, name: str = "head") -> np.ndarray:
        """The gathered fp16 output of a link after the last step."""
        import torch
        from .gather import unpack
        torch.cuda.synchronize()
        return unpack(self.outs[name].tensor.cpu().numpy(), self.chain.epoch())

    def close(self) -> None:
        self.chain.close()
        self.gg.close()
        self.file.close()
