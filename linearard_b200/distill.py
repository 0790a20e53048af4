"""End-to-end self-distillation step with the KL operator dropped in.

This is the training step of LinearARD's ``train.py:165-465`` for the
end-to-end benchmark configuration: a random-init LLaMA2-7B architecture
(32 layers, hidden 4096, 32 heads, d = 128, vocab 32000), uniform random
token ids, seq 16384, batch 1 per GPU; a frozen teacher with native RoPE and
a student with linear-scaled RoPE (factor 8) and LoRA r = 16 on q/k/v; the
loss is the Q/Q, K/K and V/V relation KL of every layer, normalised as
``train.py:380-410`` does; DDP over NCCL all-reduces the LoRA gradients.

What differs from the reference driver, in mechanism only:

* q/k/v are captured by an attention function registered with transformers
  (as ``record_qkv_attention``, ``train.py:109-145``) but kept as the views
  the attention layer produced: no ``.contiguous()`` copies
  (``attn_kl_align_grouped`` reads strided inputs in place);
* the 3·L relation losses are one grouped call instead of 3·L calls;
* LoRA is a small module written here (peft is not in this image): base
  weight frozen, ``A`` Kaiming-uniform, ``B`` zero, scale ``alpha / r``,
  no dropout (peft's defaults for these fields, ``train.py:271-273``);
* the model is ``LlamaModel`` without the LM head: the logits-KL term is off
  by default in the reference (``lam_l = 0``), so logits are not computed.

    python -m linearard_b200.distill [--layers 32] [--seq 16384] [--steps 3]
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m linearard_b200.distill

Prints one JSON line on rank 0 (tokens/s over all ranks, ms per step).
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch
import torch.distributed as dist
import torch.nn as nn

from .attention_KL import attn_kl_align_grouped

_ACTIVE = None   # the Capture the registered attention function records into


class Capture:
    """Per-layer q, k, v of one forward pass ([B, H, T, D] views)."""

    def __init__(self):
        self.q, self.k, self.v = {}, {}, {}

    def __enter__(self):
        global _ACTIVE
        _ACTIVE = self
        return self

    def __exit__(self, *exc):
        global _ACTIVE
        _ACTIVE = None

    def record(self, layer, q, k, v):
        self.q[layer], self.k[layer], self.v[layer] = q, k, v


def register_capture_attention(name="lkl_capture"):
    """Register an attention implementation that records q, k, v (after
    RoPE, as the reference hook sees them) and then runs SDPA."""
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    def capture_attention(module, query, key, value, attention_mask, **kwargs):
        if _ACTIVE is not None:
            _ACTIVE.record(module.layer_idx, query, key, value)
        return sdpa_attention_forward(module, query, key, value, attention_mask, **kwargs)

    ALL_ATTENTION_FUNCTIONS.register(name, capture_attention)
    return name


class LoRALinear(nn.Module):
    """y = base(x) + (x A^T B^T) * alpha / r, base frozen."""

    def __init__(self, base: nn.Linear, r: int, alpha: float):
        super().__init__()
        self.base = base
        for p in self.base.parameters():
            p.requires_grad_(False)
        dev, dt = base.weight.device, base.weight.dtype
        self.lora_A = nn.Parameter(torch.empty(r, base.in_features, device=dev, dtype=dt))
        self.lora_B = nn.Parameter(torch.zeros(base.out_features, r, device=dev, dtype=dt))
        nn.init.kaiming_uniform_(self.lora_A, a=math.sqrt(5))
        self.scale = alpha / r

    def forward(self, x):
        return self.base(x) + (x @ self.lora_A.t() @ self.lora_B.t()) * self.scale


def add_qkv_lora(model, r: int, alpha: float):
    for p in model.parameters():
        p.requires_grad_(False)
    for layer in model.layers:
        att = layer.self_attn
        att.q_proj = LoRALinear(att.q_proj, r, alpha)
        att.k_proj = LoRALinear(att.k_proj, r, alpha)
        att.v_proj = LoRALinear(att.v_proj, r, alpha)
    return [p for p in model.parameters() if p.requires_grad]


def llama_config(layers, hidden, heads, intermediate, vocab, seq, rope, attn):
    from transformers import LlamaConfig
    cfg = LlamaConfig(vocab_size=vocab, hidden_size=hidden, intermediate_size=intermediate,
                      num_hidden_layers=layers, num_attention_heads=heads,
                      num_key_value_heads=heads, max_position_embeddings=max(seq, 4096),
                      rope_parameters=rope)
    cfg._attn_implementation = attn
    cfg.use_cache = False
    return cfg


def build_models(args, device, seed=0):
    """Teacher (native RoPE, frozen) and student (same weights, linear RoPE x
    factor, LoRA on q/k/v), random init in bf16 on `device`."""
    from transformers import LlamaModel
    attn = register_capture_attention()
    base_rope = {"rope_type": "default", "rope_theta": args.rope_theta}
    student_rope = {"rope_type": "linear", "factor": args.rope_factor,
                    "rope_theta": args.rope_theta}
    torch.manual_seed(seed)
    old = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(device):
            teacher = LlamaModel(llama_config(args.layers, args.hidden, args.heads,
                                              args.intermediate, args.vocab, args.seq,
                                              base_rope, attn))
            student = LlamaModel(llama_config(args.layers, args.hidden, args.heads,
                                              args.intermediate, args.vocab, args.seq,
                                              student_rope, attn))
    finally:
        torch.set_default_dtype(old)
    student.load_state_dict(teacher.state_dict())
    teacher.eval()
    for p in teacher.parameters():
        p.requires_grad_(False)
    lora = add_qkv_lora(student, args.lora_r, args.lora_alpha)
    student.train()
    return teacher, student, lora


def relation_loss(cap_s: Capture, cap_t: Capture, layers, attn_mask=None, sm_scale=None):
    """train.py:380-410: per layer KL_Q/denom + KL_K/denom + KL_V/denom, mean
    over layers, denom = valid tokens x Hq.  One grouped call for all of them."""
    items = []
    for l in layers:
        for s, t in ((cap_s.q[l], cap_t.q[l]), (cap_s.k[l], cap_t.k[l]),
                     (cap_s.v[l], cap_t.v[l])):
            items.append((s, s, t, t))
    kl = attn_kl_align_grouped(items, attn_mask=attn_mask, causal=True, sm_scale_s=sm_scale,
                               sm_scale_t=sm_scale)
    qs = cap_s.q[layers[0]]
    if attn_mask is None:
        denom = qs.shape[0] * qs.shape[1] * qs.shape[2]
    else:
        denom = attn_mask.sum().clamp_min(1) * qs.shape[1]
    return kl.sum() / denom / max(1, len(layers))


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--intermediate", type=int, default=11008)
    ap.add_argument("--vocab", type=int, default=32000)
    ap.add_argument("--seq", type=int, default=16384)
    ap.add_argument("--rope-theta", type=float, default=10000.0)
    ap.add_argument("--rope-factor", type=float, default=8.0)
    ap.add_argument("--lora-r", type=int, default=16)
    ap.add_argument("--lora-alpha", type=float, default=32.0)
    ap.add_argument("--lr", type=float, default=1e-4)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=1)
    return ap.parse_args(argv)


def main(argv=None):
    from torch.nn.parallel import DistributedDataParallel as DDP
    args = parse(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    teacher, student, lora = build_models(args, dev, seed=0)
    model = DDP(student, device_ids=[local]) if world > 1 else student
    opt = torch.optim.AdamW(lora, lr=args.lr)
    layers = list(range(args.layers))
    g = torch.Generator(device=dev).manual_seed(1000 + rank)

    def step(marks=None):
        def mark():
            if marks is not None:
                marks.append(torch.cuda.Event(enable_timing=True))
                marks[-1].record()
        ids = torch.randint(0, args.vocab, (1, args.seq), device=dev, generator=g)
        mark()
        with torch.no_grad(), Capture() as cap_t:
            teacher(input_ids=ids, use_cache=False)
        mark()
        with Capture() as cap_s:
            model(input_ids=ids, use_cache=False)
        mark()
        loss = relation_loss(cap_s, cap_t, layers)
        mark()
        loss.backward()                      # DDP all-reduces the LoRA gradients
        mark()
        opt.step()
        opt.zero_grad(set_to_none=True)
        mark()
        out = loss.detach()
        if world > 1:
            dist.all_reduce(out)
            out /= world
        return out

    for _ in range(args.warmup):
        step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        loss = step()
    e1.record()
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev)
    # one more step with events between its phases (reported, not in the timing)
    marks = []
    step(marks)
    torch.cuda.synchronize()
    names = ("teacher_forward", "student_forward", "kl_forward_grouped",
             "backward_kl_model_and_lora_allreduce", "optimizer")
    phases = {n: marks[i].elapsed_time(marks[i + 1]) for i, n in enumerate(names)}
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    if rank == 0:
        ms_step = float(ms.item())
        print(json.dumps({
            "metric": "self-distillation step tokens/s (LLaMA2-7B arch, random init, LoRA r=%d "
                      "on q/k/v, Q/Q+K/K+V/V KL over all layers)" % args.lora_r,
            "value": args.seq * world / (ms_step / 1e3), "unit": "tokens/s", "n_gpus": world,
            "ms_per_step": ms_step, "steps": args.steps, "warmup": args.warmup,
            "config": {"layers": args.layers, "hidden": args.hidden, "heads": args.heads,
                       "seq_len": args.seq, "batch_per_gpu": 1, "rope_factor": args.rope_factor,
                       "lora_r": args.lora_r, "parallelism": f"ddp{world}"},
            "loss": float(loss.item()),
            "phase_ms_rank0": phases,
            "peak_mem_gb": torch.cuda.max_memory_allocated(dev) / 2**30,
        }), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
