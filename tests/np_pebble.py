"""Independent float64 numpy forward of the Pebble-25M architecture, written
from the layer equations rather than from the oracle's code.  Used only to check
that the C oracle's structure (layer pattern, in_proj split, conv window, SSD,
gate-then-norm, RoPE, KV cache, tied head) is right; agreement is to float32
rounding, not bitwise."""
import numpy as np

H, V, I, NL, NH, HD = 608, 2048, 2432, 8, 8, 76
DS, DI, MP, MH, DXBC = 128, 1216, 64, 19, 1472


def _rms(x, w, eps):
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * w


def _silu(x):
    return x / (1.0 + np.exp(-x))


def _softplus(x):
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))


def _erf_as(x):
    # Abramowitz & Stegun 7.1.26 (the approximation the reference uses)
    a1, a2, a3, a4, a5, p = 0.254829592, -0.284496736, 1.421413741, -1.453152027, 1.061405429, 0.3275911
    s = np.where(x < 0, -1.0, 1.0)
    ax = np.abs(x)
    t = 1.0 / (1.0 + p * ax)
    return s * (1.0 - ((((a5 * t + a4) * t + a3) * t + a2) * t + a1) * t * np.exp(-ax * ax))


def _gelu(x):
    return 0.5 * x * (1.0 + _erf_as(x / np.sqrt(2.0)))


def _rope(x, pos):
    half = HD // 2
    x = x.reshape(NH, HD).copy()
    i = np.arange(half)
    ang = pos / (10000.0 ** (2.0 * i / HD))
    c, s = np.cos(ang), np.sin(ang)
    a, b = x[:, :half].copy(), x[:, half:].copy()
    x[:, :half] = a * c - b * s
    x[:, half:] = a * s + b * c
    return x.reshape(-1)


class NpPebble:
    def __init__(self, w, max_ctx=2048):
        self.w = {k: np.asarray(v, np.float64) for k, v in w.items()}
        self.ctx = max_ctx
        self.reset()

    def reset(self):
        self.pos = 0
        self.conv = {l: np.zeros((DXBC, 4)) for l in range(NL) if l % 4 < 3}
        self.ssm = {l: np.zeros((MH, MP, DS)) for l in range(NL) if l % 4 < 3}
        self.k = {l: np.zeros((self.ctx, H)) for l in range(NL) if l % 4 == 3}
        self.v = {l: np.zeros((self.ctx, H)) for l in range(NL) if l % 4 == 3}

    def _token(self, tok):
        w = self.w
        x = w["wte.weight"][tok].copy()
        pos = self.pos
        for l in range(NL):
            p = f"blocks.{l}."
            if l % 4 < 3:
                h = _rms(x, w[p + "ln.weight"], 1e-6)
                zx = w[p + "mixer.in_proj.weight"] @ h
                z, xbc, dt = zx[:DI], zx[DI:DI + DXBC], zx[DI + DXBC:]
                cs = self.conv[l]
                cs[:, :3] = cs[:, 1:].copy()
                cs[:, 3] = xbc
                cw = w[p + "mixer.conv1d.weight"].reshape(DXBC, 4)
                u = _silu((cs * cw).sum(1) + w[p + "mixer.conv1d.bias"])
                xs, bs, cc = u[:DI].reshape(MH, MP), u[DI:DI + DS], u[DI + DS:]
                dtv = _softplus(dt + w[p + "mixer.dt_bias"])
                da = np.exp(dtv * -np.exp(w[p + "mixer.A_log"]))
                st = self.ssm[l]
                st[:] = st * da[:, None, None] + (xs * dtv[:, None])[:, :, None] * bs[None, None, :]
                y = st @ cc + w[p + "mixer.D"][:, None] * xs
                y = y.reshape(-1) * _silu(z)
                y = _rms(y, w[p + "mixer.norm.weight"], 1e-5)
                x = x + w[p + "mixer.out_proj.weight"] @ y
            else:
                h = _rms(x, w[p + "ln1.weight"], 1e-6)
                qkv = w[p + "wqkv.weight"] @ h
                q, k, v = _rope(qkv[:H], pos), _rope(qkv[H:2 * H], pos), qkv[2 * H:]
                self.k[l][pos], self.v[l][pos] = k, v
                K = self.k[l][: pos + 1].reshape(pos + 1, NH, HD)
                Vv = self.v[l][: pos + 1].reshape(pos + 1, NH, HD)
                sc = np.einsum("hd,thd->ht", q.reshape(NH, HD), K) / np.sqrt(HD)
                sc = np.exp(sc - sc.max(1, keepdims=True))
                sc /= sc.sum(1, keepdims=True)
                ao = np.einsum("ht,thd->hd", sc, Vv).reshape(-1)
                x = x + w[p + "wo.weight"] @ ao
                h = _rms(x, w[p + "ln2.weight"], 1e-6)
                x = x + w[p + "fc2.weight"] @ _gelu(w[p + "fc1.weight"] @ h)
        self.pos += 1
        return w["wte.weight"] @ _rms(x, w["lnf.weight"], 1e-6)

    def prefill(self, toks):
        out = None
        for t in toks:
            out = self._token(int(t))
        return out

    def step(self, tok):
        return self._token(int(tok))
