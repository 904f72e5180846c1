"""Generate the golden fixtures under tests/golden/ by running the REFERENCE implementation
(imronpuji/wisp-runtime 0.1.0, Python) in the build container.

    WISP_REFERENCE=/path/to/wisp-runtime python tests/golden/make_golden.py

The reference cannot travel to the GPU box, so its outputs are frozen here as small .npz files.  The
tests compare the numpy oracle (oracle/wisp_oracle.py) against these files, which pins the oracle to
the reference; the GPU tests then compare the CUDA kernels against the pinned oracle and, where a
fixture exists, against the fixture directly.

Every fixture is produced by the reference's own public functions:
  quant_*.npz     wisp.quant.quantize / _unpack / dequant           (wisp/quant.py:17-87)
  kernels.npz     wisp.kernels.moe_decode_q4 / _q4_fast / _q3_fast    (wisp/kernels.py:115-322, run under
                  TRITON_INTERPRET=1 exactly like the reference tests/test_kernels.py) and the
                  dequant+einsum oracle of tests/test_kernels.py:10-18
  rope.npz        wisp.kernels.rope_decode and HF apply_rotary_pos_emb (tests/test_fastattn.py:16-27)
  norm.npz        patched Qwen3MoeRMSNorm (wisp/model.py:94-107) and the HF original
  moe_block.npz   wisp.moe.PagedMoEBlock.forward on a CPU stand-in cache (decode branch N<=4 and the
                  per-expert branch N>4, wisp/moe.py:62-137), 4/3/2-bit
  gptoss.npz      wisp.gptoss.PagedGptOssBlock.forward on a CPU stand-in cache (wisp/gptoss.py:111-143)
  attn.npz        the graph decoder's masked GQA SDPA (wisp/graphdec.py:169-175)
  cache_trace.npz decisions of wisp.cache_core.CacheCore (wisp/cache_core.py:15-149) on seeded
                  operation sequences: ensure / split / admit / acquire / resized under lru, wsa and
                  static, with the resulting slots, page-ins, residency and statistics

    python tests/golden/make_golden.py [generator ...]   (default: all; e.g. `cache_trace`)
"""

import os
import sys

os.environ["TRITON_INTERPRET"] = "1"
REF = os.environ.get("WISP_REFERENCE")
if not REF:
    sys.exit("set WISP_REFERENCE to the reference source tree (the directory holding its wisp/ package)")
sys.path.insert(0, REF)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.nn.functional as F  # noqa: E402

from wisp import quant  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def u16(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def gen_quant():
    for group, n in ((128, 2048 * 3), (32, 2048)):
        rec = {}
        g = torch.Generator().manual_seed(1234 + group)
        w32 = torch.randn(3, n, generator=g) * 0.02
        # a few groups with special structure: constant (scale clamps to 1e-5) and wide range
        w32[0, :group] = 0.0125
        w32[1, group : 2 * group] = torch.linspace(-3.0, 5.0, group)
        wbf = w32.to(torch.bfloat16)
        rec["w_f32"] = w32.numpy()
        rec["w_bf16"] = u16(wbf)
        for bits in (16, 8, 4, 3, 2):
            for tag, w in (("f32", w32), ("bf16", wbf)):
                buf = quant.quantize(w, bits, group)
                rec[f"buf_b{bits}_{tag}"] = buf.numpy()
                rec[f"deq_b{bits}_{tag}"] = u16(quant.dequant(buf[None], n, bits, group)[0])
                if bits < 16:
                    ncode = (3 * n * bits) // 8
                    rec[f"codes_b{bits}_{tag}"] = quant._unpack(buf[None, :ncode], bits)[0].to(torch.uint8).numpy()
            rec[f"nbytes_b{bits}"] = np.int64(quant.expert_nbytes(n, bits, group))
        np.savez_compressed(os.path.join(OUT, f"quant_g{group}.npz"), n=np.int64(n), group=np.int64(group), **rec)
    # the reference's own known answers (tests/test_quant.py:37-40) at the Qwen3-30B-A3B expert size
    known = {f"b{b}": quant.expert_nbytes(1572864, b, 128) for b in (16, 8, 4, 3, 2)}
    np.savez_compressed(os.path.join(OUT, "nbytes_qwen3.npz"), **{k: np.int64(v) for k, v in known.items()})


def gen_kernels():
    from wisp.kernels import moe_decode_q3_fast, moe_decode_q4, moe_decode_q4_fast

    rec = {}
    H, I, E, k = 256, 128, 6, 3
    n = H * I
    for bits, seed in ((4, 0), (3, 2)):
        torch.manual_seed(seed)
        w3 = torch.randn(E, 3, n) * 0.05
        pool = torch.stack([quant.quantize(w3[e].to(torch.bfloat16), bits, 128) for e in range(E)])
        slots = torch.tensor([4, 1, 2] if bits == 4 else [2, 5, 1])
        x = torch.randn(H).to(torch.bfloat16)
        w = torch.softmax(torch.randn(k), 0)
        meta = torch.cat([slots.float(), w.float()])
        W = quant.dequant(pool[slots], n, bits, 128).float()
        gm, um, dm = W[:, 0].view(-1, I, H), W[:, 1].view(-1, I, H), W[:, 2].view(-1, H, I)
        a = F.silu(gm @ x.float()) * (um @ x.float())
        exp = (torch.einsum("khi,ki->kh", dm, a) * w.float()[:, None]).sum(0)
        rec[f"pool_b{bits}"] = pool.numpy()
        rec[f"slots_b{bits}"] = slots.numpy()
        rec[f"x_b{bits}"] = u16(x)
        rec[f"w_b{bits}"] = w.numpy()
        rec[f"ref_b{bits}"] = exp.numpy()
        if bits == 4:
            rec["q4_v1"] = u16(moe_decode_q4(pool, slots, x, w, n, H, I))
            rec["q4_fast"] = u16(moe_decode_q4_fast(pool, meta, x, k, n, H, I))
        else:
            rec["q3_fast"] = u16(moe_decode_q3_fast(pool, meta, x, k, n, H, I))
    np.savez_compressed(os.path.join(OUT, "kernels.npz"), H=H, I=I, E=E, k=k, **rec)


def gen_rope_norm():
    from transformers.models.qwen3_moe import modeling_qwen3_moe as m

    from wisp.kernels import rope_decode

    torch.manual_seed(0)
    D, Hq, Hk = 128, 32, 4
    q = torch.randn(1, 1, Hq, D).to(torch.bfloat16).transpose(1, 2)
    k = torch.randn(1, 1, Hk, D).to(torch.bfloat16).transpose(1, 2)
    cos = torch.randn(1, 1, D).to(torch.bfloat16)
    sin = torch.randn(1, 1, D).to(torch.bfloat16)
    qr, kr = m.apply_rotary_pos_emb(q, k, cos, sin)
    qo, ko = rope_decode(q, k, cos, sin)
    np.savez_compressed(
        os.path.join(OUT, "rope.npz"),
        q=u16(q.contiguous()),
        k=u16(k.contiguous()),
        cos=u16(cos),
        sin=u16(sin),
        q_hf=u16(qr.contiguous()),
        k_hf=u16(kr.contiguous()),
        q_wisp=u16(qo),
        k_wisp=u16(ko),
    )

    from wisp.model import patch_fast_norm

    rec = {}
    torch.manual_seed(0)
    for H in (2048, 128):
        nm = m.Qwen3MoeRMSNorm(H, 1e-6).to(torch.bfloat16)
        nm.weight.data = (torch.randn(H) * 0.3 + 1).to(torch.bfloat16)
        x = (torch.randn(3, H) * 2).to(torch.bfloat16)
        orig = m.Qwen3MoeRMSNorm.forward
        ref = orig(nm, x)
        patch_fast_norm()
        got = nm(x)
        m.Qwen3MoeRMSNorm.forward = orig
        m.Qwen3MoeRMSNorm._wisp_patched = False
        rec[f"x_{H}"], rec[f"w_{H}"] = u16(x), u16(nm.weight.data)
        rec[f"hf_{H}"], rec[f"wisp_{H}"] = u16(ref), u16(got)
    np.savez_compressed(os.path.join(OUT, "norm.npz"), **rec)


class _FakeStore:
    def __init__(self, n, bits, group):
        self.n, self.bits, self.group = n, bits, group


class _FakeCache:
    """CPU stand-in for ExpertCache (slot == key), the pattern of the reference tests/test_gptoss.py:27-40."""

    decode_on_load = False

    def __init__(self, rows, n, bits, group):
        self.rows, self.store = rows, _FakeStore(n, bits, group)

    def ensure(self, keys):
        return list(keys)

    def weights_batched(self, idx):
        return quant.dequant(self.rows[idx], self.store.n, self.store.bits, self.store.group)

    def weights(self, slots):
        return list(self.weights_batched(torch.as_tensor(slots)).unbind(0))


def gen_moe_block():
    from transformers import Qwen3MoeConfig

    from wisp.moe import PagedMoEBlock, Runtime

    rec = {}
    H, I, E, k, G = 256, 128, 16, 4, 128
    n = H * I
    cfg = Qwen3MoeConfig(
        hidden_size=H,
        moe_intermediate_size=I,
        num_experts=E,
        num_experts_per_tok=k,
        norm_topk_prob=True,
        num_hidden_layers=1,
        num_attention_heads=2,
        num_key_value_heads=1,
        head_dim=32,
        vocab_size=32,
    )
    for bits in (4, 3, 2):
        torch.manual_seed(10 + bits)
        w3 = torch.randn(E, 3, n) * 0.05
        rows = torch.stack([quant.quantize(w3[e].to(torch.bfloat16), bits, G) for e in range(E)])
        gate = torch.nn.Linear(H, E, bias=False).to(torch.bfloat16)
        with torch.no_grad():
            gate.weight.normal_(0, 0.05)
        rt = Runtime(None, fused=0)
        rt.fused = 0
        rt.cache = _FakeCache(rows, n, bits, G)
        blk = PagedMoEBlock(gate, 0, rt, cfg)
        rec[f"pool_b{bits}"] = rows.numpy()
        rec[f"gate_b{bits}"] = u16(gate.weight.data)
        for N in (1, 4, 16):
            x = torch.randn(1, N, H).to(torch.bfloat16)
            with torch.no_grad():
                out, logits = blk(x)
            rec[f"x_b{bits}_N{N}"] = u16(x[0])
            rec[f"out_b{bits}_N{N}"] = u16(out[0])
            rec[f"logits_b{bits}_N{N}"] = u16(logits)
            # the reference's own routing (wisp/moe.py:67-72), ties broken by torch.topk
            rw = F.softmax(logits, dim=1, dtype=torch.float32)
            rw, sel = torch.topk(rw, k, dim=-1)
            rw = (rw / rw.sum(dim=-1, keepdim=True)).to(torch.bfloat16)
            rec[f"sel_b{bits}_N{N}"] = sel.numpy()
            rec[f"rw_b{bits}_N{N}"] = u16(rw)
    np.savez_compressed(os.path.join(OUT, "moe_block.npz"), H=H, I=I, E=E, k=k, G=G, **rec)


def gen_gptoss():
    from transformers import GptOssConfig
    from transformers.models.gpt_oss.modeling_gpt_oss import GptOssMLP

    from wisp.gptoss import PagedGptOssBlock, expert_w3

    class FakeRT:
        def __init__(self):
            self.stats = dict(layer_calls=0, gpu_experts=0)
            self.recorder, self.chunk, self.cache = None, 4, None

    rec = {}
    torch.manual_seed(1)
    cfg = GptOssConfig(
        hidden_size=256,
        intermediate_size=256,
        num_hidden_layers=1,
        num_local_experts=8,
        num_experts_per_tok=4,
        num_attention_heads=2,
        num_key_value_heads=1,
        head_dim=32,
        vocab_size=50,
    )
    ref = GptOssMLP(cfg).to(torch.bfloat16)
    with torch.no_grad():
        for p in ref.parameters():
            p.normal_(0, 0.05)
    E, H, I, bits, G = 8, 256, 256, 4, 128
    rows = torch.stack(
        [
            quant.quantize(expert_w3(ref.experts.gate_up_proj[e].data, ref.experts.down_proj[e].data), bits, G)
            for e in range(E)
        ]
    )
    rt = FakeRT()
    rt.cache = _FakeCache(rows, H * I, bits, G)
    blk = PagedGptOssBlock(ref.router, 0, rt, cfg, device="cpu")
    blk.gub.copy_(ref.experts.gate_up_proj_bias.data)
    blk.db.copy_(ref.experts.down_proj_bias.data)
    rec.update(
        pool=rows.numpy(),
        router_w=u16(ref.router.weight.data),
        router_b=u16(ref.router.bias.data),
        gub=u16(blk.gub),
        db=u16(blk.db),
    )
    for N in (1, 5):
        x = torch.randn(1, N, H).to(torch.bfloat16)
        with torch.no_grad():
            got, sc = blk(x)
        rec[f"x_N{N}"], rec[f"out_N{N}"] = u16(x[0]), u16(got[0])
    np.savez_compressed(os.path.join(OUT, "gptoss.npz"), H=H, I=I, E=E, k=4, G=G, **rec)


def gen_attn():
    torch.manual_seed(3)
    Hq, Hk, D, T, pos = 32, 4, 128, 64, 37
    q = torch.randn(1, Hq, 1, D).to(torch.bfloat16)
    kc = torch.randn(1, Hk, T, D).to(torch.bfloat16)
    vc = torch.randn(1, Hk, T, D).to(torch.bfloat16)
    ar = torch.arange(T)
    mask = (ar <= pos).view(1, 1, 1, -1)
    o = F.scaled_dot_product_attention(
        q.reshape(1, Hk, Hq // Hk, D).float(), kc.float(), vc.float(), attn_mask=mask, scale=D**-0.5
    )
    np.savez_compressed(
        os.path.join(OUT, "attn.npz"), q=u16(q[0, :, 0]), kc=u16(kc[0]), vc=u16(vc[0]), pos=pos, out=o.reshape(Hq, D).numpy()
    )


def gen_cache_trace():
    """Seeded operation sequences run through the reference CacheCore; every result is recorded so a
    reimplementation can be replayed against them.  Keys are layer * E + expert with Zipf-biased
    experts (a few hot ones), k distinct experts per call."""
    import json

    from wisp.cache_core import CacheCore

    L, E, k = 4, 32, 4
    cases = [
        dict(name="lru", nslots=24, policy="lru", decay=0.9995, n_static=0, admit_after=2.0, steps=500, seed=11),
        dict(name="wsa", nslots=24, policy="wsa", decay=0.97, n_static=0, admit_after=2.0, steps=500, seed=12),
        # decay 0.5: the growing increment passes 1e100 after ~333 steps, so the renormalisation runs
        dict(name="wsa_renorm", nslots=20, policy="wsa", decay=0.5, n_static=0, admit_after=1.5, steps=800, seed=13),
        dict(name="static", nslots=24, policy="static", decay=0.99, n_static=8, admit_after=2.0, steps=400, seed=14),
        dict(name="lru_tight", nslots=9, policy="lru", decay=0.9995, n_static=0, admit_after=2.0, steps=400, seed=15),
    ]
    out = []
    for c in cases:
        rng = np.random.default_rng(c["seed"])
        pop = 1.0 / np.arange(1, E + 1) ** 1.1
        pop /= pop.sum()
        perm = [rng.permutation(E) for _ in range(L)]
        core = CacheCore(c["nslots"], c["policy"], c["decay"], c["n_static"], c["admit_after"])
        ops = []
        if c["n_static"]:
            keys = [int(l * E + perm[l][0]) for l in range(L)] + [int(l * E + perm[l][1]) for l in range(L)]
            keys = keys[: c["n_static"]]
            ops.append(dict(op="preload", keys=keys, res=[list(p) for p in core.preload(keys)]))
        for t in range(c["steps"]):
            l = t % L
            ex = rng.choice(E, k, replace=False, p=pop)
            keys = [int(l * E + perm[l][e]) for e in ex]
            r = rng.random()
            try:
                if r < 0.6:
                    slots, loads = core.ensure(keys)
                    ops.append(dict(op="ensure", keys=keys, res=[[int(s) for s in slots], [list(map(int, p)) for p in loads]]))
                elif r < 0.8:
                    hk, hs, mk = core.split(keys)
                    ops.append(dict(op="split", keys=keys, res=[list(map(int, hk)), list(map(int, hs)), list(map(int, mk))]))
                elif r < 0.9:
                    prot = sorted({int(s) for s in rng.choice(core.nslots, 3, replace=False)})
                    s = core.admit(keys[0], set(prot))
                    ops.append(dict(op="admit", keys=keys[:1], prot=prot, res=-1 if s is None else int(s)))
                elif r < 0.985 or c["n_static"]:
                    prot = sorted({int(s) for s in rng.choice(core.nslots, 2, replace=False)})
                    if core.lookup(keys[0]) is None:
                        s = core.acquire(keys[0], set(prot))
                        ops.append(dict(op="acquire", keys=keys[:1], prot=prot, res=int(s)))
                    else:
                        ops.append(dict(op="lookup", keys=keys[:1], res=int(core.lookup(keys[0]))))
                else:
                    n2 = int(rng.integers(max(k, c["nslots"] // 2), c["nslots"] + 8))
                    core, loads = core.resized(n2)
                    ops.append(dict(op="resized", n=n2, res=[list(map(int, p)) for p in loads]))
            except RuntimeError as e:
                ops.append(dict(op="error", keys=keys, msg=str(e)))
                break
            ops[-1]["resident"] = sorted([int(a), int(b)] for a, b in core.key2slot.items())
            ops[-1]["stats"] = dict(core.stats)
        out.append(dict(case=c, ops=ops))
    np.savez_compressed(os.path.join(OUT, "cache_trace.npz"), trace=np.array(json.dumps(out)))


GENERATORS = dict(quant=gen_quant, kernels=gen_kernels, rope_norm=gen_rope_norm, moe_block=gen_moe_block,
                  gptoss=gen_gptoss, attn=gen_attn, cache_trace=gen_cache_trace)

if __name__ == "__main__":
    for name in sys.argv[1:] or list(GENERATORS):
        GENERATORS[name]()
    for f in sorted(os.listdir(OUT)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(OUT, f)))
