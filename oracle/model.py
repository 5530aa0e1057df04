"""The operators of oracle.numpy_ref composed into the decode step the graph runs: embedding,
27 layers (layer 0 dense, the rest MoE), the head and greedy argmax.

TEST INFRASTRUCTURE (see oracle/__init__.py for who may import it).

The composition follows the reference's operator order (fleet/graph_plan.py:416-602):
  embed; per layer: norm1 + qkva, mla_prep (cache append at the step row), mla_attend,
  mla_merge_uv, o_proj + residual; layer 0: norm2, gate_up, SwiGLU, down + residual;
  MoE layers: router (norm2 folded in), w13, w2 (SwiGLU prologue), combine + residual;
  head: final norm + lm_head, argmax -> tokens[pos + 1].

Weights are read through ``get(name)`` (whole tensor) and ``get_expert(name, e)`` (one expert's
slice of W13/W2) returning float32 arrays of BF16 values, so a test can feed the oracle from
device tensors without copying the 31 GB model. Keys are the packed layout of
fleet/pack_weights.py (``W_ukT_l`` is transposed back to W_uk here).
"""
import numpy as np

from oracle import numpy_ref as R
from oracle.detmath import F32


class OracleModel:
    def __init__(self, dims, get, get_expert=None, *, softmax_scale, split=32, eps=1e-6,
                 layers=None, head=True, logit_bias=None, fp8=None):
        self.d = dims
        self.get = get
        self.get_expert = get_expert or (lambda name, e: get(name)[e])
        self.scale = softmax_scale
        self.split = split
        self.eps = eps
        self.layers = dims.L if layers is None else layers
        self.head = head
        self.logit_bias = logit_bias          # {layer: [E] FP32} injected routing (config 3)
        # FP8 experts: fp8(l, e) -> (W13q [2I, H], s13 [2], W2q [H, I], s2), E4M3 codes (uint8) and
        # the expert's gate, up and down scales; the experts then run numpy_ref.linear_fp8
        self.fp8 = fp8

    def W_uk(self, l):
        return np.ascontiguousarray(self.get(f"W_ukT_{l}").transpose(0, 2, 1))

    @staticmethod
    def gate_up(w):
        """The packed W13 / W_gu interleave gate and up rows (row 2i gate i, 2i+1 up i); the
        reference's arithmetic reads [gate rows; up rows]."""
        return np.concatenate([w[0::2], w[1::2]], axis=0)

    def attention(self, l, x_res, cache, cos, sin, pos, rec):
        d = self.d
        h, qkva = R.linear_norm(x_res, self.get(f"w_norm1_{l}"), self.get(f"W_qkva_{l}"), self.eps)
        c_row, k_row, ql_nope, q_pe = R.mla_prep(qkva, self.get(f"w_kv_norm_{l}"), self.W_uk(l),
                                                 cos[pos], sin[pos], nh=d.NH, d_n=d.D_N, d_r=d.D_R,
                                                 d_c=d.D_C, eps=self.eps)
        c_kv, k_pe = cache[f"c_kv_{l}"], cache[f"k_pe_{l}"]
        c_kv[pos], k_pe[pos] = c_row, k_row
        partials = R.mla_attend(ql_nope, q_pe, c_kv, k_pe, pos, self.scale, split=self.split)
        attn = R.mla_merge_uv(partials, self.get(f"W_uv_{l}"), pos, split=self.split)
        x_attn = R.linear_residual(attn, self.get(f"W_o_{l}"), x_res)
        if rec is not None:
            rec.update({f"L{l}.norm1": h, f"L{l}.qkva": qkva, f"L{l}.c_kv": c_row, f"L{l}.k_pe": k_row,
                        f"L{l}.ql_nope": ql_nope, f"L{l}.q_pe": q_pe, f"L{l}.partials": partials,
                        f"L{l}.attn": attn, f"L{l}.x_res_attn": x_attn})
        return x_attn

    def dense_mlp(self, x_res, rec):
        d = self.d
        h = R.rmsnorm(x_res, self.get("w_norm2_0"), self.eps)
        mid, act, out = R.dense_mlp(h, self.gate_up(self.get("W_gu_0")), self.get("W_down_0"), x_res, d.I_DENSE)
        if rec is not None:
            rec.update({"L0.norm2": h, "L0.mid": mid, "L0.act": act, "L0.layer_out": out})
        return out

    def moe(self, l, x_res, rec):
        d = self.d
        bias = None if self.logit_bias is None else self.logit_bias.get(l)
        h, logits, topk_w, routing, mask = R.moe_router_norm(
            x_res, self.get(f"w_norm2_{l}"), self.get(f"W_gate_{l}"), eps=self.eps, topk=d.TOPK,
            n_experts=d.E, forced=tuple(range(d.E, d.E_TOTAL)), logit_bias=bias)
        n_slots = d.N_SLOTS
        mid = np.full((n_slots, 2 * d.I_MOE), np.nan, F32)
        out8 = np.full((n_slots, d.H), np.nan, F32)
        for s in range(int(mask[-1])):
            e = int(mask[s])
            if self.fp8 is not None:
                w13q, s13, w2q, s2 = self.fp8(l, e)
                mid[s] = np.concatenate([R.linear_fp8(h, w13q[0::2], s13[0]), R.linear_fp8(h, w13q[1::2], s13[1])])
                act = R.swiglu_act(mid[s], d.I_MOE)
                out8[s] = R.linear_fp8(act, w2q, s2)
                continue
            mid[s] = R.linear(h, self.gate_up(self.get_expert(f"W13_{l}", e)))
            act = R.swiglu_act(mid[s], d.I_MOE)
            out8[s] = R.linear(act, self.get_expert(f"W2_{l}", e))
        out = R.moe_combine(out8, topk_w, x_res)
        if rec is not None:
            rec.update({f"L{l}.norm2": h, f"L{l}.router_logits": logits, f"L{l}.topk_w": topk_w,
                        f"L{l}.routing": routing, f"L{l}.mask": mask, f"L{l}.mid": mid,
                        f"L{l}.out8": out8, f"L{l}.layer_out": out})
        return out

    def step(self, token, pos, cache, cos, sin, record=False):
        """One decode token at position `pos`: returns (next token, x_res after the last layer,
        record dict or None). Writes cache rows `pos` of every layer."""
        rec = {} if record else None
        x = R.embed(self.get("W_embed"), token)
        if rec is not None:
            rec["embed"] = x
        for l in range(self.layers):
            x = self.attention(l, x, cache, cos, sin, pos, rec)
            x = self.dense_mlp(x, rec) if l == 0 else self.moe(l, x, rec)
        tok = None
        if self.head:
            h, logits, tok = R.lm_head_argmax(x, self.get("w_final_norm"), self.get("W_lm"), self.eps)
            if rec is not None:
                rec.update({"head.norm": h, "head.logits": logits, "head.token": tok})
        return tok, x, rec

    def generate(self, tokens, pos0, iters, cache, cos, sin, record_last=False, on_step=None):
        """Greedy decode: iteration i reads tokens[pos0 + i] and writes tokens[pos0 + i + 1].
        Returns (ids, route_log [iters][moe layers] of the TOPK ids, last record). on_step(i, rec)
        sees every iteration's record (router probabilities, logits) as it is made."""
        ids, routes, rec = [], [], None
        for i in range(iters):
            pos = pos0 + i
            last = record_last and i == iters - 1
            tok, _, r = self.step(int(tokens[pos]), pos, cache, cos, sin, record=True)
            routes.append([r[f"L{l}.mask"][:self.d.TOPK].tolist() for l in range(1, self.layers)])
            if on_step is not None:
                on_step(i, r)
            if last:
                rec = r
            tokens[pos + 1] = tok
            ids.append(tok)
        return ids, routes, rec
