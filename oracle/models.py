"""GPT-2 and Qwen3 forward passes restated over the C restatement's ops. TEST INFRASTRUCTURE ONLY.

Each class follows the reference's CPU forward line by line (paths relative to app/architecture):
* ``Qwen3``: qwen3/cpp/qwen3_model.cpp:232-276 (+ loading :116-160, rope table :102-114)
* ``Gpt2``:  gpt2/cpp/gpt2_model.cpp:179-218 (+ loading :84-122; Conv1D weights transposed through f16, :78-82)
The op calls are the restatement's (oracle/neko_oracle.c), so for the same weights the logits are
bit-identical to the compiled reference's (checked in tests/test_oracle.py).
"""
import numpy as np

from .oracle import ACCUMULATE, F16, GELU, Restatement


def _fmt_for(cols, fmt):  # Model::formatFor (model.h:164)
    return fmt if cols % 32 == 0 else F16


class _Base:
    def __init__(self, R, shape, tensors, fmt, context):
        self.R = R if R is not None else Restatement()
        self.s = dict(shape)
        self.fmt = fmt
        self.ctx = context
        self.t = {n: np.asarray(a, np.float32) for n, a in tensors}

    def q(self, *names, transpose_f16=False):
        """Model::matrix: rows of the named tensors, concatenated, in the engine's packed format."""
        mats = []
        for n in names:
            w = self.t[n]
            if transpose_f16:  # TensorStore::toF16(name, true) then f16 -> f32
                w = np.ascontiguousarray(w.T).astype(np.float16).astype(np.float32)
            mats.append(w)
        w = np.concatenate(mats, 0)
        f = _fmt_for(w.shape[1], self.fmt)
        return f, self.R.quantize(f, w), w.shape[1]

    def mm(self, m, x, T, y, y_stride, flags, bias=None):
        f, q, K = m
        self.R.matmul(f, x, q, K, bias, y, y_stride, flags)


class Qwen3(_Base):
    def __init__(self, shape, tensors, fmt, context, R=None):
        super().__init__(R, shape, tensors, fmt, context)
        s = self.s
        C, H, KV, hd, F = s["embd"], s["heads"], s["kv_heads"], s["head_dim"], s["ff"]
        self.embed = self.q("embed_tokens.weight")
        self.normf = self.t["norm.weight"]
        self.rope = self.R.rope_table(context, hd, s["rope_theta"])
        self.layers = []
        for l in range(s["layers"]):
            p = f"layers.{l}."
            self.layers.append(dict(
                ln1=self.t[p + "input_layernorm.weight"], ln2=self.t[p + "post_attention_layernorm.weight"],
                qn=self.t[p + "self_attn.q_norm.weight"], kn=self.t[p + "self_attn.k_norm.weight"],
                wqkv=self.q(p + "self_attn.q_proj.weight", p + "self_attn.k_proj.weight", p + "self_attn.v_proj.weight"),
                wo=self.q(p + "self_attn.o_proj.weight"),
                wgu=self.q(p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight"),
                wdown=self.q(p + "mlp.down_proj.weight"),
                kc=np.zeros((context, KV * hd), np.uint16), vc=np.zeros((context, KV * hd), np.uint16)))

    def forward(self, tokens, pos0, stop_layer=None, stage=0):
        """stop_layer / stage: Model::setDebugLayers semantics (qwen3_model.cpp:237-273)."""
        R, s = self.R, self.s
        C, H, KV, hd, F = s["embd"], s["heads"], s["kv_heads"], s["head_dim"], s["ff"]
        eps = s["eps"]
        T = len(tokens)
        QW, kOff, vOff = (H + 2 * KV) * hd, H * hd, (H + KV) * hd
        f, q, _ = self.embed
        x = R.embed(f, q, C, tokens)
        for li, L in enumerate(self.layers):
            if stop_layer is not None and li >= stop_layer and not (stage and li == stop_layer):
                return x
            at = (lambda st: stop_layer is not None and stage == st and li == stop_layer)
            xn = R.rms_norm(x, L["ln1"], eps)
            if at(1):
                return xn
            qkv = np.zeros((T, QW), np.float32)
            self.mm(L["wqkv"], xn, T, qkv, QW, 0)
            if at(2):
                return qkv
            for t in range(T):
                r = qkv[t]
                r[:kOff] = R.rms_norm(r[:kOff].reshape(H, hd), L["qn"], eps).reshape(-1)
                r[kOff:vOff] = R.rms_norm(r[kOff:vOff].reshape(KV, hd), L["kn"], eps).reshape(-1)
                R.rope(r, H + KV, hd, self.rope[pos0 + t])
            if at(3):
                return qkv
            R.store_kv(qkv[:, kOff:], qkv[:, vOff:], QW, L["kc"], L["vc"], KV * hd, T, pos0)
            att = R.attention(qkv, QW, L["kc"], L["vc"], T, H, KV, hd, pos0)
            if at(4):
                return att
            self.mm(L["wo"], att, T, x, C, ACCUMULATE)
            if at(5):
                return x
            xn = R.rms_norm(x, L["ln2"], eps)
            if at(6):
                return xn
            h = np.zeros((T, 2 * F), np.float32)
            self.mm(L["wgu"], xn, T, h, 2 * F, 0)
            if at(7):
                return h
            g = R.silu_mul(h, F)
            if at(8):
                return g
            self.mm(L["wdown"], g, T, x, C, ACCUMULATE)
            if at(9):
                return x
        if stop_layer is not None:
            return x
        xn = R.rms_norm(x[T - 1:T], self.normf, eps)
        logits = np.zeros((1, s["vocab"]), np.float32)
        self.mm(self.embed, xn, 1, logits, s["vocab"], 0)
        return logits[0]


class Gpt2(_Base):
    def __init__(self, shape, tensors, fmt, context, R=None):
        super().__init__(R, shape, tensors, fmt, context)
        s = self.s
        C = s["embd"]
        self.wte = self.q("wte.weight")
        self.wpe = self.t["wpe.weight"]
        self.lnf = (self.t["ln_f.weight"], self.t["ln_f.bias"])
        self.layers = []
        for l in range(s["layers"]):
            p = f"h.{l}."
            self.layers.append(dict(
                ln1=(self.t[p + "ln_1.weight"], self.t[p + "ln_1.bias"]),
                ln2=(self.t[p + "ln_2.weight"], self.t[p + "ln_2.bias"]),
                wqkv=self.q(p + "attn.c_attn.weight", transpose_f16=True), bqkv=self.t[p + "attn.c_attn.bias"],
                wproj=self.q(p + "attn.c_proj.weight", transpose_f16=True), bproj=self.t[p + "attn.c_proj.bias"],
                wfc=self.q(p + "mlp.c_fc.weight", transpose_f16=True), bfc=self.t[p + "mlp.c_fc.bias"],
                wfc2=self.q(p + "mlp.c_proj.weight", transpose_f16=True), bfc2=self.t[p + "mlp.c_proj.bias"],
                kc=np.zeros((context, C), np.uint16), vc=np.zeros((context, C), np.uint16)))

    def forward(self, tokens, pos0, stop_layer=None, stage=0):
        """stop_layer / stage: Model::setDebugLayers semantics (gpt2_model.cpp:188-215)."""
        R, s = self.R, self.s
        C, H = s["embd"], s["heads"]
        hd, F, eps = C // H, s["ff"], s["eps"]
        T = len(tokens)
        f, q, _ = self.wte
        x = R.embed(f, q, C, tokens, self.wpe, pos0)
        for li, L in enumerate(self.layers):
            if stop_layer is not None and li >= stop_layer and not (stage and li == stop_layer):
                return x
            at = (lambda st: stop_layer is not None and stage == st and li == stop_layer)
            xn = R.layer_norm(x, *L["ln1"], eps)
            if at(1):
                return xn
            qkv = np.zeros((T, 3 * C), np.float32)
            self.mm(L["wqkv"], xn, T, qkv, 3 * C, 0, L["bqkv"])
            if at(2):
                return qkv
            R.store_kv(qkv[:, C:], qkv[:, 2 * C:], 3 * C, L["kc"], L["vc"], C, T, pos0)
            att = R.attention(qkv, 3 * C, L["kc"], L["vc"], T, H, H, hd, pos0)
            if at(3):
                return att
            self.mm(L["wproj"], att, T, x, C, ACCUMULATE, L["bproj"])
            if at(4):
                return x
            xn = R.layer_norm(x, *L["ln2"], eps)
            if at(5):
                return xn
            h = np.zeros((T, F), np.float32)
            self.mm(L["wfc"], xn, T, h, F, GELU, L["bfc"])
            if at(6):
                return h
            self.mm(L["wfc2"], h, T, x, C, ACCUMULATE, L["bfc2"])
            if at(7):
                return x
        if stop_layer is not None:
            return x
        xn = R.layer_norm(x[T - 1:T], *self.lnf, eps)
        logits = np.zeros((1, s["vocab"]), np.float32)
        self.mm(self.wte, xn, 1, logits, s["vocab"], 0)
        return logits[0]


def make(shape, tensors, fmt, context, R=None):
    cls = Qwen3 if shape["arch"] == "qwen3" else Gpt2
    return cls(shape, tensors, fmt, context, R)
