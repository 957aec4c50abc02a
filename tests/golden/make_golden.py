"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run where the reference source tree is importable (it is not needed anywhere
else):

    REFERENCE_SRC=/path/to/nari-qwen3-tts/src python tests/golden/make_golden.py

It executes the reference's own CPU code on seeded inputs and stores inputs
and outputs as small torch files next to this script:

  sampler.pt    sample_logits_stateless (model/sampling.py:127-225); the
                probability vector each row hands to torch.multinomial is
                captured too, so the oracle's filtered probabilities are pinned.
  planner.pt    PagedTalkerKV metadata (executor/talker_kv.py:403-533) and
                allocator publications over a seeded script of add / prefill /
                decode / publish / discard / remove operations.
  binding.pt    what the reference's PagedTalkerKV hands a custom
                binding_factory (executor/talker_kv.py:358-388) and every
                metadata object it plans (prepare_prefill / prepare_decode /
                prepare_capture, :485-533), recorded by a stand-in binding,
                so the drop-in binding can be replayed against exactly
                those calls without the reference installed.
  fp8.pt        quantize_fp8_weight_blocks (model/layers.py:11-25) on a
                seeded bf16 weight whose 128 x 128 blocks cover a zero block,
                an amax below the 1e-4 clamp, amax exactly 448 * 2^k, huge and
                subnormal magnitudes and ordinary N(0, 1) data.
  attention.pt  RMSNorm.forward + Qwen3TTSCodePredictor._apply_rope
                (model/layers.py:103-115, model/components.py:214-233) on
                bf16 heads, and _depth_attention (components.py:236-252) on
                KV gathered from a paged layout for decode, causal prefill
                and the code-predictor short cache.
"""

from __future__ import annotations

import os
import random
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


def _import_reference():
    src = os.environ.get("REFERENCE_SRC")
    if not src:
        raise SystemExit("set REFERENCE_SRC to the reference's src/ directory")
    sys.path.insert(0, src)
    from nari_qwen3_tts.contract import TalkerDecodeCaptureKey, TalkerPrefillCaptureKey
    from nari_qwen3_tts.executor.talker_kv import PagedTalkerKV
    from nari_qwen3_tts.model.components import Qwen3TTSCodePredictor
    from nari_qwen3_tts.model.layers import RMSNorm, quantize_fp8_weight_blocks
    from nari_qwen3_tts.model.sampling import sample_logits_stateless

    return {
        "TalkerDecodeCaptureKey": TalkerDecodeCaptureKey,
        "TalkerPrefillCaptureKey": TalkerPrefillCaptureKey,
        "PagedTalkerKV": PagedTalkerKV,
        "CP": Qwen3TTSCodePredictor,
        "RMSNorm": RMSNorm,
        "quantize_fp8": quantize_fp8_weight_blocks,
        "sample": sample_logits_stateless,
    }


# ----------------------------------------------------------------------------- sampler
def _sampler_cases() -> list[dict]:
    g = torch.Generator().manual_seed(0)
    cases = []

    def case(name, rows, vocab, *, dtype=torch.float32, temperature=0.9, top_k=50, top_p=0.95, penalty=1.05,
             seen=True, offsets=None, greedy_rows=()):
        logits = (torch.randn(rows, vocab, generator=g) * 2.0 ** 0.5).to(dtype)
        temp = torch.full((rows,), float(temperature))
        for r in greedy_rows:
            temp[r] = 0.0
        seen_mask = None
        if seen:
            ids = torch.randint(0, vocab, (rows, 64), generator=g)
            seen_mask = torch.zeros(rows, vocab, dtype=torch.bool).scatter_(1, ids, True)
        cases.append(
            {
                "name": name,
                "logits": logits,
                "temperature": temp,
                "top_k": torch.full((rows,), int(top_k), dtype=torch.int32),
                "top_p": torch.full((rows,), float(top_p)),
                "seed": torch.arange(rows, dtype=torch.long) + 1000 * len(cases),
                "offset": offsets if offsets is not None else torch.zeros(rows, dtype=torch.long),
                "repetition_penalty": torch.full((rows,), float(penalty)),
                "seen_token_mask": seen_mask,
            }
        )

    # B=8, V=3072, N(0, 2) logits, T 0.9, k 50, p 0.95, penalty 1.05 over 64 seen ids
    case("config1", 8, 3072)
    case("full_vocab_top_p", 4, 3072, top_k=0, top_p=0.9)
    case("top_k_only", 4, 3072, top_p=1.0)
    case("top_k_1", 4, 3072, top_k=1)
    case("k_above_vocab", 2, 512, top_k=4096, top_p=0.8)
    case("greedy_mixed", 6, 3072, greedy_rows=(0, 3))
    case("cp_bf16_no_seen", 8, 2048, dtype=torch.bfloat16, seen=False, top_p=1.0,
         offsets=torch.tensor([f * 512 + c * 32 for f, c in zip(range(8), range(1, 9))], dtype=torch.long))
    case("low_temperature", 4, 3072, temperature=0.3, top_p=0.7)
    case("large_offsets", 4, 3072, offsets=torch.tensor([2**40 + 7, 5 * 512 + 32, 123456789, 0], dtype=torch.long))
    return cases


def make_sampler(ref) -> dict:
    cases = _sampler_cases()
    captured: list[torch.Tensor] = []
    real_multinomial = torch.multinomial

    def recording_multinomial(probs, num_samples, *args, **kwargs):
        captured.append(probs.detach().clone())
        return real_multinomial(probs, num_samples, *args, **kwargs)

    out = []
    for c in cases:
        captured.clear()
        torch.multinomial = recording_multinomial
        try:
            tokens = ref["sample"](
                c["logits"], c["temperature"], c["top_k"], c["top_p"], c["seed"], c["offset"],
                repetition_penalty=c["repetition_penalty"], seen_token_mask=c["seen_token_mask"],
            )
        finally:
            torch.multinomial = real_multinomial
        c = dict(c)
        c["tokens"] = tokens.clone()
        c["multinomial_probs"] = list(captured)
        out.append(c)
    return {"cases": out}


# ----------------------------------------------------------------------------- planner
def make_planner(ref) -> dict:
    rng = random.Random(7)
    total_pages, page_size, scratch = 22, 4, 6
    kv = ref["PagedTalkerKV"](
        num_layers=1, num_kv_heads=2, num_qo_heads=4, head_dim=8, total_pages=total_pages, page_size=page_size,
        scratch_page_count=scratch, workspace_bytes=1024, device=torch.device("cpu"), dtype=torch.float32,
        binding_factory=lambda **kwargs: kwargs,
    )
    live: list[str] = []
    next_id = 0
    steps = []
    slot = 0
    for step in range(48):
        # churn: remove a request or admit a new one
        if live and rng.random() < 0.2:
            rid = live.pop(rng.randrange(len(live)))
            kv.remove_request(rid)
            steps.append({"op": "remove", "rid": rid})
        if len(live) < 5 and rng.random() < 0.6:
            rid = f"r{next_id}"
            next_id += 1
            kv.add_request(rid)
            live.append(rid)
            steps.append({"op": "add", "rid": rid})
        if not live:
            continue
        prefill = rng.random() < 0.35
        rows = rng.sample(live, k=rng.randint(1, min(4, len(live))))
        capture_rows = 4
        if prefill:
            advances = tuple(rng.randint(1, 14) for _ in rows)
            token_capacity = 24
            key = ref["TalkerPrefillCaptureKey"](capture_rows, token_capacity, None)
            context = kv.create_prefill(key, slot=slot)
            try:
                pubs = kv.prepare_prefill(context, key, tuple(rows), advances)
            except Exception as error:  # allocation failure is part of the contract
                steps.append({"op": "prefill", "rows": rows, "advances": list(advances), "error": type(error).__name__,
                              "capture_rows": capture_rows, "token_capacity": token_capacity})
                continue
        else:
            advances = (1,) * len(rows)
            token_capacity = capture_rows
            key = ref["TalkerDecodeCaptureKey"](capture_rows)
            context = kv.create_decode(key, slot=slot)
            try:
                pubs = kv.prepare_decode(context, key, tuple(rows))
            except Exception as error:
                steps.append({"op": "decode", "rows": rows, "advances": list(advances), "error": type(error).__name__,
                              "capture_rows": capture_rows, "token_capacity": token_capacity})
                continue
        md = context["metadata"]
        publish = [rng.random() < 0.85 for _ in rows]
        steps.append(
            {
                "op": "prefill" if prefill else "decode",
                "rows": rows,
                "advances": list(advances),
                "capture_rows": capture_rows,
                "token_capacity": token_capacity,
                "publish": publish,
                "qo_indptr": None if md.qo_indptr is None else md.qo_indptr.tolist(),
                "paged_kv_indptr": md.paged_kv_indptr.tolist(),
                "paged_kv_indices": md.paged_kv_indices.tolist(),
                "paged_kv_last_page_len": md.paged_kv_last_page_len.tolist(),
                "position_ids": md.position_ids.tolist(),
                "write_pages": md.write_pages.tolist(),
                "write_offsets": md.write_offsets.tolist(),
                "publication_pages": [list(p.page_indices) for p in pubs],
            }
        )
        for p, ok in zip(pubs, publish, strict=True):
            (p.publish if ok else p.discard)()
    final = {rid: {"pages": list(kv.state(rid).page_indices), "length": kv.state(rid).sequence_length}
             for rid in live}
    return {"total_pages": total_pages, "page_size": page_size, "scratch": scratch, "steps": steps, "final": final,
            "free_pages": kv.allocator.free_pages}


# ----------------------------------------------------------------------------- attention
def make_attention(ref) -> dict:
    g = torch.Generator().manual_seed(3)
    out: dict = {}
    # QK norm + RoPE on bf16 heads (talker shapes, positions up to ~4k)
    tokens, hq, hkv, d, theta, eps = 6, 16, 8, 128, 1.0e6, 1e-6
    q = torch.randn(tokens, hq, d, generator=g).to(torch.bfloat16)
    k = torch.randn(tokens, hkv, d, generator=g).to(torch.bfloat16)
    qw = (1.0 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    kw = (1.0 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    pos = torch.tensor([0, 1, 17, 511, 2047, 4095], dtype=torch.long)
    qn = ref["RMSNorm"](d, eps=eps)
    kn = ref["RMSNorm"](d, eps=eps)
    with torch.no_grad():
        qn.weight.copy_(qw.float())
        kn.weight.copy_(kw.float())
        # RMSNorm computes in fp32 and casts back to the input dtype, like the kernel's rounding point
        q_normed = qn(q)
        k_normed = kn(k)
        q_rot = ref["CP"]._apply_rope(q_normed.unsqueeze(0), pos.unsqueeze(0), rope_theta=theta)[0]
        k_rot = ref["CP"]._apply_rope(k_normed.unsqueeze(0), pos.unsqueeze(0), rope_theta=theta)[0]
    out["norm_rope"] = {"q": q, "k": k, "q_weight": qw, "k_weight": kw, "positions": pos, "eps": eps,
                        "theta": theta, "q_out": q_rot, "k_out": k_rot}

    # paged layout (config-1 shapes, fewer rows): decode and causal prefill through _depth_attention
    page_size, total_pages = 16, 24
    cache = torch.randn(total_pages, 2, page_size, hkv, d, generator=g).to(torch.bfloat16).float()
    lens = [16, 37, 100, 129]
    perm = torch.randperm(total_pages, generator=g).tolist()
    indptr, indices, last = [0], [], []
    for n in lens:
        pages = (n + page_size - 1) // page_size
        indices.extend(perm[:pages])
        perm = perm[pages:]
        indptr.append(len(indices))
        last.append(n % page_size or page_size)
    qd = torch.randn(len(lens), hq, d, generator=g)
    decode_out = []
    for b, n in enumerate(lens):
        pages = torch.tensor(indices[indptr[b]: indptr[b + 1]])
        kk = cache[pages, 0].reshape(-1, hkv, d)[:n].transpose(0, 1).unsqueeze(0)
        vv = cache[pages, 1].reshape(-1, hkv, d)[:n].transpose(0, 1).unsqueeze(0)
        mask = torch.ones(1, 1, 1, n, dtype=torch.bool)
        o = ref["CP"]._depth_attention(qd[b].unsqueeze(0).unsqueeze(2), kk, vv, mask)
        decode_out.append(o[0, :, 0])
    qo_lens = [3, 1, 20, 64]
    qo_indptr = [0]
    for x in qo_lens:
        qo_indptr.append(qo_indptr[-1] + x)
    qp = torch.randn(qo_indptr[-1], hq, d, generator=g)
    prefill_out = torch.zeros_like(qp)
    for b, n in enumerate(lens):
        pages = torch.tensor(indices[indptr[b]: indptr[b + 1]])
        kk = cache[pages, 0].reshape(-1, hkv, d)[:n].transpose(0, 1).unsqueeze(0)
        vv = cache[pages, 1].reshape(-1, hkv, d)[:n].transpose(0, 1).unsqueeze(0)
        ql = qo_lens[b]
        qi = torch.arange(ql).view(-1, 1)
        kj = torch.arange(n).view(1, -1)
        mask = (kj <= n - ql + qi).view(1, 1, ql, n)
        qq = qp[qo_indptr[b]: qo_indptr[b + 1]].transpose(0, 1).unsqueeze(0)
        o = ref["CP"]._depth_attention(qq, kk, vv, mask)
        prefill_out[qo_indptr[b]: qo_indptr[b + 1]] = o[0].transpose(0, 1)
    out["paged"] = {
        "cache": cache.to(torch.bfloat16), "page_size": page_size, "indptr": torch.tensor(indptr, dtype=torch.int32),
        "indices": torch.tensor(indices, dtype=torch.int32), "last_page_len": torch.tensor(last, dtype=torch.int32),
        "q_decode": qd, "decode_out": torch.stack(decode_out), "qo_indptr": torch.tensor(qo_indptr, dtype=torch.int32),
        "q_prefill": qp, "prefill_out": prefill_out,
    }

    # code-predictor short cache: rows 5, capacity 16, D 64, cache_pos 6 (7 visible)
    rows, cap, d_cp, cache_pos = 5, 16, 64, 6
    kc = torch.randn(rows, cap, hkv, d_cp, generator=g)
    vc = torch.randn(rows, cap, hkv, d_cp, generator=g)
    qc = torch.randn(rows, hq, d_cp, generator=g)
    key_positions = torch.arange(cache_pos + 1)
    mask = (key_positions.unsqueeze(0) <= torch.tensor([[cache_pos]])).view(1, 1, 1, cache_pos + 1)
    o = ref["CP"]._depth_attention(qc.unsqueeze(2), kc[:, : cache_pos + 1].transpose(1, 2),
                                   vc[:, : cache_pos + 1].transpose(1, 2), mask)
    out["short_cache"] = {"q": qc, "k_cache": kc, "v_cache": vc, "length": cache_pos + 1, "out": o[:, :, 0]}
    return out


# ----------------------------------------------------------------------------- binding
_META_FIELDS = ("qo_indptr", "paged_kv_indptr", "paged_kv_indices", "paged_kv_last_page_len", "position_ids",
                "write_pages", "write_offsets", "padding_pages", "reuse_attention_plan")


def make_binding(ref) -> dict:
    """Drive the reference PagedTalkerKV through a prefill, three published
    decode steps and a capture warm-up with a recording binding factory."""

    import dataclasses

    calls: list[dict] = []
    factories: list[dict] = []

    class Recorder:
        def __init__(self, **kwargs) -> None:
            self.index = len(factories)
            factories.append({
                "keys": sorted(kwargs),
                "scalars": {k: v for k, v in kwargs.items() if isinstance(v, (int, float, bool)) or v is None},
                "storage_shape": tuple(kwargs["storage"].shape),
                "workspace_bytes": int(kwargs["workspace"].numel()),
                "workspace_dtype": str(kwargs["workspace"].dtype),
                "shared_plan_state": type(kwargs["shared_plan_state"]).__name__,
                "dtype": str(kwargs["dtype"]),
            })

        def plan(self, metadata) -> None:
            fields = [f.name for f in dataclasses.fields(metadata)]
            entry = {"binding": self.index, "fields": fields}
            for name in fields:
                value = getattr(metadata, name)
                entry[name] = value.clone() if isinstance(value, torch.Tensor) else value
            calls.append(entry)

    kv = ref["PagedTalkerKV"](num_layers=2, num_kv_heads=8, num_qo_heads=16, head_dim=128, total_pages=96,
                              page_size=16, scratch_page_count=12, workspace_bytes=64 << 20,
                              device=torch.device("cpu"), dtype=torch.bfloat16, binding_factory=Recorder)
    for rid in ("a", "b", "c"):
        kv.add_request(rid)
    pkey = ref["TalkerPrefillCaptureKey"](4, 192, None)
    pre = kv.create_prefill(pkey, slot=0)
    for pub in kv.prepare_prefill(pre, pkey, ("a", "b", "c"), (40, 7, 100)):
        pub.publish()
    dkey = ref["TalkerDecodeCaptureKey"](4)
    dec = kv.create_decode(dkey, slot=0)
    for _ in range(3):
        for pub in kv.prepare_decode(dec, dkey, ("a", "b", "c")):
            pub.publish()
    kv.abort(kv.prepare_capture(dec, dkey))
    return {"factories": factories, "calls": calls, "metadata_fields": list(_META_FIELDS)}


def make_fp8(ref) -> dict:
    """A [256, 768] bf16 weight: six 128 x 128 blocks per block row, each a different regime."""

    g = torch.Generator().manual_seed(11)
    w = torch.randn(256, 768, generator=g)
    blocks = w.view(2, 128, 6, 128)
    blocks[0, :, 0] = 0.0                                   # all zero: amax clamped to 1e-4
    blocks[0, :, 1] *= 2e-5                                 # amax below the clamp
    blocks[0, :, 2] = blocks[0, :, 2].clamp(-50, 50)        # amax exactly 448 * 2^-3 (a power-of-two scale)
    blocks[0, 7, 2, 9] = -56.0
    blocks[0, :, 3] *= 1e30                                 # huge magnitudes
    blocks[0, :, 4] *= 1e-38                                # bf16 subnormals: quantise to zero
    blocks[0, :, 5] = blocks[0, :, 5].clamp(-400, 400)      # amax exactly 448
    blocks[0, 100, 5, 3] = 448.0
    blocks[1] *= torch.logspace(-3, 3, 6).view(1, 6, 1)    # ordinary data over six decades
    weight = w.to(torch.bfloat16).contiguous()
    q, scales = ref["quantize_fp8"](weight)
    return {"weight": weight, "q": q.view(torch.uint8).clone(), "scales": scales.clone()}


MAKERS = {
    "sampler": make_sampler,
    "planner": make_planner,
    "attention": make_attention,
    "binding": make_binding,
    "fp8": make_fp8,
}


def main() -> None:
    """Writes every fixture, or only those named on the command line (e.g. ``make_golden.py fp8``)."""

    ref = _import_reference()
    names = sys.argv[1:] or list(MAKERS)
    for name in names:
        torch.save(MAKERS[name](ref), HERE / f"{name}.pt")
        print(f"{name}.pt", (HERE / f"{name}.pt").stat().st_size, "bytes")


if __name__ == "__main__":
    main()
