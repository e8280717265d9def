"""Generate the golden fixtures under tests/golden/ from the reference implementation itself.

Run in the build container, where the reference source tree is mounted (pass its path with
``--ref``): ``python tests/golden/make_golden.py --ref <reference checkout>``. The reference package
is imported under the alias ``sisa_ref`` and only its pure-PyTorch (CPU) code paths run. The
resulting ``*.pt`` files are committed; the tests read them without the reference.

Cases (all seeded):
  attn_case.pt   sisa_attention_torch in fp64 on prepared inputs, output and every input gradient
  prep_case.pt   SISAAttention._prepare (torch glue) of a seeded sublayer, and the fused projection
                 (concat_fused_weights + F.linear) of the same input
  lce_case.pt    reference_linear_cross_entropy in fp64 with ignored rows, loss and gradients
  model_case.pt  tiny SISAForCausalLM (torch backend, fp64): state dict, loss, logits, a few grads,
                 greedy generate() tokens and the cached-decode logits
  known.pt       preset parameter counts, fused layouts for H = 8, 12, 16
  ckpt_case.pt   a tiny model saved by the reference's save_pretrained (safetensors and .bin bytes), its
                 logits, and its convert_state_dict of paper-layout and wrapper-prefixed keys
"""
from __future__ import annotations

import argparse
import importlib.util
import sys
from pathlib import Path

import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent


def import_reference(ref: Path):
    src = ref / "src" / "sisa"
    spec = importlib.util.spec_from_file_location("sisa_ref", src / "__init__.py",
                                                  submodule_search_locations=[str(src)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["sisa_ref"] = mod
    spec.loader.exec_module(mod)
    return mod


def proj_inputs(B, L, H, seed):
    """Seeded inputs with the benchmark distributions (same generator order as the oracle's helper)."""
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(B, L, H * 64, generator=gen)
    k = torch.randn(B, L, H * 64, generator=gen)
    v = torch.randn(B, L, H * 64, generator=gen)
    bm = torch.randn(B, L, H * 32, generator=gen)
    cm = torch.randn(B, L, H * 32, generator=gen)
    th = torch.randn(B, L, H * 16, generator=gen) * 0.2
    a = torch.randn(B, L, H, generator=gen) * 0.45 - 2.5
    z = torch.randn(B, L, H, generator=gen) * 0.45 + 1.0
    return q, k, v, bm, cm, th, a, z


def attn_case(ref):
    fn = ref.functional
    B, L, H = 2, 77, 2
    q, k, v, bm, cm, th, a, z = proj_inputs(B, L, H, seed=11)
    t = lambda x, w: x.view(B, L, H, w).transpose(1, 2).double()   # noqa: E731
    g = torch.cumsum(-F.softplus(a.double().transpose(1, 2)), 2)
    phi = torch.cumsum(t(th, 16), 2)
    c = fn.rotate_pairs(t(cm, 32), phi)
    b = fn.rotate_pairs(t(bm, 32), phi)
    Fg = torch.cumsum(F.logsigmoid(z.double()).transpose(1, 2), 2)
    lam = F.softplus(torch.tensor([-0.7, 0.4], dtype=torch.float64))
    ins = dict(q=t(q, 64), k=t(k, 64), v=t(v, 64), c=c, b=b, g=g, lam=lam, F=Fg)
    xs = {n: x.clone().requires_grad_(True) for n, x in ins.items()}
    o = fn.sisa_attention_torch(xs["q"], xs["k"], xs["v"], xs["c"], xs["b"], xs["g"], xs["lam"], xs["F"],
                                block_q=32)
    dout = torch.randn(o.shape, generator=torch.Generator().manual_seed(5), dtype=torch.float64)
    gr = torch.autograd.grad(o, list(xs.values()), dout)
    out = {"inputs": {n: x.detach() for n, x in ins.items()}, "dout": dout, "o": o.detach()}
    out["grads"] = {"d" + n: gg for n, gg in zip(xs.keys(), gr)}
    return out


def prep_case(ref):
    cfg = ref.SISAConfig(vocab_size=97, d_model=128, n_layer=1, n_head=2, d_ff=64, attn_impl="torch",
                         zero_init_c=False)
    torch.manual_seed(3)
    att = ref.SISAAttention(cfg)
    gen = torch.Generator().manual_seed(4)
    with torch.no_grad():
        att.theta_proj.weight.copy_(torch.randn(att.theta_proj.weight.shape, generator=gen) * 0.2)
        att.alpha_proj.bias.copy_(torch.rand(2, generator=gen) * 3.0 - 4.0)
        att.forget_proj.bias.copy_(torch.rand(2, generator=gen) * 3.0)
    x = torch.randn(2, 70, 128, generator=gen)
    with torch.no_grad():
        q, k, v, c, b, g, fgate, phi = att._prepare(x)
        from sisa_ref.kernels.fused_prep import concat_fused_weights, fused_layout

        W, bias = concat_fused_weights(att.W_Q.weight, att.W_K.weight, att.W_V.weight, att.W_B.weight,
                                       att.W_C.weight, att.theta_proj.weight, att.alpha_proj.weight,
                                       att.alpha_proj.bias)
        proj = F.linear(x, W, bias)
        zl = att._forget_logits(x)
    return dict(proj=proj, z=zl, n_head=2, layout=fused_layout(2),
                ref=dict(q=q, k=k, v=v, c=c, b=b, g=g, F=fgate, phi=phi))


def lce_case(ref):
    from sisa_ref.kernels.linear_ce import reference_linear_cross_entropy

    gen = torch.Generator().manual_seed(21)
    N, D, V = 37, 64, 101
    h = torch.randn(N, D, generator=gen, dtype=torch.float64).requires_grad_(True)
    w = (torch.randn(V, D, generator=gen, dtype=torch.float64) * 0.3).requires_grad_(True)
    labels = torch.randint(0, V, (N,), generator=gen)
    labels[[3, 10, 11]] = -100
    loss = reference_linear_cross_entropy(h, w, labels)
    dh, dw = torch.autograd.grad(loss, [h, w])
    return dict(hidden=h.detach(), weight=w.detach(), labels=labels, loss=loss.detach(), dh=dh, dw=dw)


def model_case(ref):
    cfg = ref.SISAConfig(vocab_size=97, d_model=128, n_layer=2, n_head=2, d_ff=96, attn_impl="torch")
    torch.manual_seed(7)
    model = ref.SISAForCausalLM(cfg)
    gen = torch.Generator().manual_seed(8)
    with torch.no_grad():   # switch every score term on
        for layer in model.layers:
            at = layer.attn
            at.W_C.weight.copy_(torch.randn(at.W_C.weight.shape, generator=gen) * 0.08)
            at.theta_proj.weight.copy_(torch.randn(at.theta_proj.weight.shape, generator=gen) * 0.2)
            at.alpha_proj.bias.copy_(torch.rand(2, generator=gen) * 3.0 - 4.0)
            at.forget_proj.bias.copy_(torch.rand(2, generator=gen) * 3.0)
            at.lambda_raw.copy_(torch.rand(2, generator=gen) * 2.0 - 0.5)
    state = {k: v.detach().clone() for k, v in model.state_dict().items()}
    ids = torch.randint(0, 97, (2, 40), generator=gen)
    m64 = model.double()
    out = m64(ids, labels=ids)
    out.loss.backward()
    grads = {n: p.grad.detach().clone() for n, p in m64.named_parameters()
             if n in ("embed.weight", "layers.0.attn.lambda_raw", "layers.1.attn.alpha_proj.bias",
                      "layers.0.attn.theta_proj.weight", "layers.1.attn.forget_proj.weight")}
    with torch.no_grad():
        prompt = ids[:, :12]
        gen_tokens = m64.generate(prompt, max_new_tokens=8)
        cache = ref.generation.SISACache()
        pre = m64(prompt, cache=cache, logits_to_keep=1).logits[:, -1]
        step = m64(gen_tokens[:, 12:13], cache=cache, logits_to_keep=1).logits[:, -1]
    return dict(config=cfg.to_dict(), state_dict=state, ids=ids, loss=out.loss.detach(),
                logits=out.logits.detach(), grads=grads, prompt=prompt, generated=gen_tokens,
                prefill_logits=pre, step_logits=step)


def known(ref):
    counts = {name: ref.SISAConfig.preset(name).num_parameters() for name in ref.PRESETS}
    from sisa_ref.kernels.fused_prep import fused_layout

    return dict(param_counts=counts, layouts={h: fused_layout(h) for h in (8, 12, 16)},
                state_dict_keys=sorted(ref.SISAForCausalLM(ref.SISAConfig(
                    vocab_size=97, d_model=128, n_layer=2, n_head=2, d_ff=96)).state_dict().keys()))


def paper_layout(state_dict, prefix=""):
    """A state dict renamed to the paper training code's layout: attention parameters directly under
    ``layers.{i}``, norms and SwiGLU as compiled submodules (``._orig_mod.``), an optional wrapper prefix."""
    out = {}
    for key, value in state_dict.items():
        parts = key.split(".")
        if len(parts) > 3 and parts[0] == "layers" and parts[2] == "attn":
            del parts[2]
        elif len(parts) > 3 and parts[0] == "layers" and parts[2] in ("attn_norm", "ffn_norm", "ffn"):
            parts.insert(3, "_orig_mod")
        elif parts[0] == "final_norm":
            parts.insert(1, "_orig_mod")
        out[prefix + ".".join(parts)] = value
    return out


def ckpt_case(ref):
    """Files written by the reference's save_pretrained (both formats), its logits, and its key
    conversion of paper-layout and wrapper-prefixed keys."""
    import tempfile

    cfg = ref.SISAConfig(vocab_size=61, d_model=32, n_layer=2, n_head=2, d_ff=40, d_state=8, attn_impl="torch")
    torch.manual_seed(21)
    model = ref.SISAForCausalLM(cfg)
    gen = torch.Generator().manual_seed(22)
    with torch.no_grad():
        for layer in model.layers:
            layer.attn.W_C.weight.copy_(torch.randn(layer.attn.W_C.weight.shape, generator=gen) * 0.1)
    model.eval()
    ids = torch.randint(0, 61, (2, 24), generator=gen)
    with torch.no_grad():
        logits = model(ids).logits
    files = {}
    for safe, name in ((True, "model.safetensors"), (False, "pytorch_model.bin")):
        with tempfile.TemporaryDirectory() as tmp:
            model.save_pretrained(tmp, safe_serialization=safe)
            files[name] = (Path(tmp) / name).read_bytes()
            files["config.json"] = (Path(tmp) / "config.json").read_bytes()
    keys = list(model.state_dict().keys())
    odd = ["module.layers.0.W_Q.weight", "_orig_mod.module.layers.1.lambda_raw", "module._orig_mod.embed.weight",
           "layers.3.ffn._orig_mod.w_up.weight", "layers.10.W_Obias", "layers.2.alpha_proj", "layers.x.W_Q.weight",
           "module", "_orig_mod.", "final_norm._orig_mod.weight", "layers.0.attn.W_B.weight", "layers.0.W_Z.weight"]
    key_map = {}
    for prefix in ("", "module.", "_orig_mod.", "module._orig_mod."):
        src = [prefix + k for k in paper_layout(dict.fromkeys(keys, torch.zeros(1)))]
        conv = ref.convert_state_dict(dict.fromkeys(src, torch.zeros(1)))
        key_map.update(zip(src, conv))
    for k in odd:
        key_map[k] = next(iter(ref.convert_state_dict({k: torch.zeros(1)})))
    inferred = ref.checkpoint.infer_config_from_state_dict(paper_layout(model.state_dict(), "module."))
    return dict(files=files, ids=ids, logits=logits, key_map=key_map, inferred=inferred.to_dict(),
                state_dict_keys=keys)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the reference checkout (read-only)")
    ap.add_argument("--only", nargs="*", help="write only these cases")
    args = ap.parse_args(argv)
    ref = import_reference(Path(args.ref))
    torch.set_num_threads(4)
    for name, fn in (("attn_case", attn_case), ("prep_case", prep_case), ("lce_case", lce_case),
                     ("model_case", model_case), ("known", known), ("ckpt_case", ckpt_case)):
        if args.only and name not in args.only:
            continue
        torch.save(fn(ref), HERE / f"{name}.pt")
        print("wrote", name)


if __name__ == "__main__":
    main()
