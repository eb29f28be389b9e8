"""Whole-model greedy decoding on the end-to-end configuration, token for token.

Model: 22 TinyLlama-shaped layers (hidden 2048, intermediate 5632, 32/4 heads
of 64, vocabulary 32000), seeded random-init bf16 weights (norm weights 1),
sink + window cache of 4 + 1024, RMSNorm eps 1e-5, RoPE theta 10000; a
2048-token prompt of uniform random ids prefilled in the reference's chunks of
n_sink + W = 1028 and 1020 tokens, then 512 greedy tokens.

The checker is the reference's own code path run on a B200: its kernels
(embedding, RMSNorm, cuBLAS / GEMV matmul, RoPE, attention, add,
fused_silu_mul, bf16_to_fp32, argmax) compiled from its sources and driven in
the order of Model::forward and Engine::run_generation (oracle/ref_model.py).
Its kernels are bf16 only, so this runs in bf16.

What identity can be asked for: both sides round every kernel's output to
bf16 (the LM head's logits too, src/model.cu:125-130), and the two sides sum
in different orders (cuBLAS and the reference GEMV against this library's
tcgen05 tiles and weight stream), so a few per cent of the values of each
layer differ by one bf16 unit.  After 22 layers the logits differ by a few
bf16 units (at logits near 3.4 a unit is 1/64), and with 32000 random logits
the two largest are that close, or exactly tied, at several per cent of the
steps; there no implementation short of a bit-identical copy of cuBLAS's
summation order can promise the reference's pick.  So, with both models fed
the same tokens (the reference's: teacher forcing), the test measures at every
step the logit error band (max over the vocabulary of |ours - reference|)
and asserts:
  * every step whose reference top-2 gap exceeds twice that step's band picks
    the reference's token: every mismatch is a near-tie the band explains;
  * the logits stay within 5e-2 of the largest logit at every step (a guard
    against gross errors), and their median band against the reference is at
    most twice that of a control: this library against itself with another
    fp32 summation order in its decode attention, i.e. how far summation order
    alone moves this model's logits (measured: 0.084 against the reference,
    0.0845 for the control);
  * free-running generation (each side feeding back its own tokens) agrees
    with the reference up to its first divergence, which is such a near-tie.
Batch 16 has no counterpart in the single-sequence reference
(include/kv_cache.h:7): each of 16 sequences decoded together must equal its
own batch-1 run token for token, all 512 tokens."""
import numpy as np
import pytest
import torch

import orininfer_b200 as ob
from oracle import oracle as O
from orininfer_b200 import weights as Wt
from orininfer_b200.layer import Decoder

pytestmark = pytest.mark.gpu

N_SINK, WINDOW, PROMPT, NEW = 4, 1024, 2048, 512
CHUNK = N_SINK + WINDOW


def synthetic_device_model(dev, seed=0, dtype=torch.bfloat16):
    """Seeded random-init weights in the reference's tensor names, made on the
    device (QKV/O/MLP/embedding/LM head ~ N(0, 0.02^2), norms 1)."""
    cfg = dict(Wt.TINYLLAMA)
    H, IM, V = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
    KVD = cfg["num_key_value_heads"] * cfg["head_dim"]
    QD = cfg["num_attention_heads"] * cfg["head_dim"]
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    shape = {"embed_tokens": (V, H), "lm_head": (V, H), "q_proj": (QD, H), "k_proj": (KVD, H),
             "v_proj": (KVD, H), "o_proj": (H, QD), "gate_proj": (IM, H), "up_proj": (IM, H),
             "down_proj": (H, IM)}
    t = {}
    for name in Wt.reference_tensor_names(cfg["num_hidden_layers"]):
        if name.endswith("norm.weight"):
            dim = cfg["head_dim"] if ("q_norm" in name or "k_norm" in name) else H
            t[name] = torch.ones(dim, dtype=dtype, device=dev)
            continue
        key = next(k for k in shape if k in name)
        t[name] = (torch.randn(shape[key], generator=gen, device=dev) * 0.02).to(dtype)
    return t, cfg


def _prompt(seed, V):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, V, (PROMPT,), generator=g).tolist()


@pytest.fixture(scope="module")
def e2e():
    from oracle.ref_model import RefModel

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    tensors, cfg = synthetic_device_model(dev)
    prompt = _prompt(0, cfg["vocab_size"])
    ref = RefModel(tensors, cfg, dev, n_sink=N_SINK, window=WINDOW)
    ref_tokens, ref_logits = ref.generate(prompt, NEW, keep_logits=True)
    del ref
    torch.cuda.empty_cache()
    ours = Decoder(tensors, cfg, dev, n_sink=N_SINK, window=WINDOW, max_tokens=CHUNK)
    yield dict(tensors=tensors, cfg=cfg, prompt=prompt, ref_tokens=ref_tokens,
               ref_logits=ref_logits, ours=ours, dev=dev)
    del ours
    torch.cuda.empty_cache()


def _top2_gap(row: torch.Tensor) -> float:
    v = torch.topk(row, 2).values
    return float(v[0] - v[1])


def _forced(ours, prompt, forced, steps, dev):
    """Our decoder fed `forced` tokens; yields (step, picked token, fp32 logits
    as the reference forms them: f32(round16(h . W)))."""
    ids = torch.tensor(prompt, dtype=torch.int32, device=dev)
    for pos in range(0, len(prompt), CHUNK):
        tok = ours.step(ids[pos:pos + CHUNK], pos)
    one = torch.empty(1, dtype=torch.int32, device=dev)
    for i in range(steps):
        if i > 0:
            one.fill_(forced[i - 1])
            tok = ours.step(one, len(prompt) + i - 1)
        pick = int(tok.item())
        yield i, pick, ob.linear(ours.xn[:1], ours.lm_head, epilogue="f32")[0]


def test_teacher_forced_tokens_match_the_reference_outside_near_ties(e2e):
    """Besides the reference, a control: the same library and weights with the
    decode attention unsplit (one CTA sweeps all keys instead of 17 key
    splits merged afterwards), i.e. the same arithmetic in another fp32
    summation order.  Its logit band against this library's default run
    measures how far this 22-layer random-weight model moves under summation
    order alone; the band against the reference is compared with it."""
    ours, prompt, R, RL = e2e["ours"], e2e["prompt"], e2e["ref_tokens"], e2e["ref_logits"]
    ctrl = Decoder(e2e["tensors"], e2e["cfg"], e2e["dev"], n_sink=N_SINK, window=WINDOW,
                   max_tokens=CHUNK)
    no_split = torch.empty(16, dtype=torch.uint8, device=e2e["dev"])
    for layer in ctrl.layers:
        layer.workspace = no_split
    agree, unexplained, worst_rel, bands, ctrl_bands = 0, [], 0.0, [], []
    runs = zip(_forced(ours, prompt, R, NEW, e2e["dev"]), _forced(ctrl, prompt, R, NEW, e2e["dev"]))
    for (i, pick, lg), (_, _, lg_c) in runs:
        # the fused LM-head argmax picks exactly the reference sampler's token
        # of this library's own logits (ties broken the reference's way)
        assert pick == O.argmax_key_order(lg.cpu().numpy()), f"step {i}"
        ref_row = RL[i]
        band = float((lg - ref_row).abs().max())
        bands.append(band)
        ctrl_bands.append(float((lg - lg_c).abs().max()))
        worst_rel = max(worst_rel, band / float(ref_row.abs().max()))
        gap = _top2_gap(ref_row)
        if pick == R[i]:
            agree += 1
        elif gap > 2 * band:
            unexplained.append((i, pick, R[i], gap, band))
    del ctrl
    torch.cuda.empty_cache()
    bands, ctrl_bands = np.array(bands), np.array(ctrl_bands)
    print(f"\nteacher-forced: {agree}/{NEW} picks equal the reference's; logit band against "
          f"the reference median {np.median(bands):.4f}, max {bands.max():.4f} (normwise "
          f"{worst_rel:.3e}); against this library with unsplit decode attention median "
          f"{np.median(ctrl_bands):.4f}, max {ctrl_bands.max():.4f}")
    assert not unexplained, f"mismatches outside the logit error band: {unexplained[:5]}"
    # a gross-error guard (a wrong layer or position moves logits by O(1)),
    # not a precision claim: 22 bf16 layers of random weights amplify
    # summation-order differences to a few per cent of the logits
    assert worst_rel <= 5e-2
    # the distance to the reference is the model's own sensitivity to fp32
    # summation order (measured ratio ~1), not an error of this library
    assert np.median(bands) <= 2.0 * np.median(ctrl_bands)
    assert agree >= 0.9 * NEW


def test_free_running_tokens_agree_until_a_near_tie(e2e):
    ours, prompt, R, RL = e2e["ours"], e2e["prompt"], e2e["ref_tokens"], e2e["ref_logits"]
    mine = ours.generate(prompt, NEW)
    assert len(mine) == NEW
    first = next((i for i in range(NEW) if mine[i] != R[i]), None)
    if first is None:
        print("\nfree-running: 512/512 tokens identical to the reference")
        return
    # until the divergence both sides were fed the same tokens
    for i, pick, lg in _forced(ours, prompt, R, first + 1, e2e["dev"]):
        pass
    assert pick == mine[first]
    band = float((lg - RL[first]).abs().max())
    gap = _top2_gap(RL[first])
    print(f"\nfree-running: the first {first} tokens are identical; at step {first} the "
          f"reference's two largest logits differ by {gap:.5f}, this library's logits differ "
          f"from the reference's by at most {band:.5f}")
    assert gap <= 2 * band, (first, gap, band)


def test_batch16_equals_batch1_token_for_token(e2e):
    tensors, cfg, dev, ours = e2e["tensors"], e2e["cfg"], e2e["dev"], e2e["ours"]
    B = 16
    prompts = [_prompt(100 + b, cfg["vocab_size"]) for b in range(B)]
    single = [ours.generate(p, NEW) for p in prompts]
    batch = Decoder(tensors, cfg, dev, n_sink=N_SINK, window=WINDOW, max_tokens=CHUNK, batch=B)
    got = batch.generate_batch(prompts, NEW)
    ob.device_check()
    for b in range(B):
        assert got[b] == single[b], (b, next(i for i in range(NEW) if got[b][i] != single[b][i]))
    assert batch.stats["decode_steps"] == NEW - 1
    print(f"\nbatch 16: {B * NEW} tokens identical to the batch-1 runs; batched decode "
          f"{batch.stats['decode_ms'] / (NEW - 1):.3f} ms per step (eager)")
