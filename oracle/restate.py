"""numpy restatement of FlowEdge's policy-sampling hot path (the parity oracle).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).  Every function cites the
reference file:line it restates (paths relative to the reference repository).
Arithmetic follows the reference's fp32 CPU path: float32 storage, float64
GroupNorm statistics, float32 matmuls (numpy's BLAS reassociates the sums,
which moves results by ~1e-6 relative; parity tests allow for it).

Parity of this restatement is pinned against the reference's own compiled
core (oracle/_ref/liboracle.so) on the committed golden fixtures in
tests/golden/ (see tests/test_oracle_golden.py).
"""

from __future__ import annotations

import math

import numpy as np

F32 = np.float32


# --------------------------------------------------------------------------
# elementwise ops (src/core/kernels/cpu/kernels_scalar.cc)


def mish(x):
    """x * tanh(softplus(x)), softplus = max(x,0) + log1p(exp(-|x|)) (kernels_scalar.cc:83-87)."""
    x = np.asarray(x, F32)
    sp = np.maximum(x, F32(0)) + np.log1p(np.exp(-np.abs(x)))
    return (x * np.tanh(sp)).astype(F32)


def silu(x):
    """x / (1 + exp(-x)) (kernels_scalar.cc:69-73)."""
    x = np.asarray(x, F32)
    return (x / (F32(1) + np.exp(-x))).astype(F32)


def softplus(x):
    """max(x,0) + log1p(exp(-|x|)) (kernels_scalar.cc:75-81)."""
    x = np.asarray(x, F32)
    return (np.maximum(x, F32(0)) + np.log1p(np.exp(-np.abs(x)))).astype(F32)


def rmsnorm(x, weight, eps=1e-5):
    """Row RMSNorm, fp32 sum of squares (kernels_scalar.cc:48-60)."""
    x = np.asarray(x, F32)
    ss = np.sum(x * x, axis=-1, keepdims=True, dtype=F32)
    scale = F32(1) / np.sqrt(ss / F32(x.shape[-1]) + F32(eps))
    return (x * scale * weight).astype(F32)


# --------------------------------------------------------------------------
# Diffusion Policy U-Net ops (src/core/kernels/diffusion_ops.cc)


def conv1d(x, w, b, stride=1, padding=None):
    """x [IC][L] -> [OC][L_out]; zero padding, PyTorch cross-correlation.

    diffusion_ops.cc:82-175 (padding = k/2 for the U-Net convs, 1 for the
    stride-2 downsample, diffusion.cc:741-751, 860-862)."""
    oc, ic, k = w.shape
    if padding is None:
        padding = k // 2
    length = x.shape[1]
    out_len = (length + 2 * padding - k) // stride + 1
    xp = np.zeros((ic, length + 2 * padding), F32)
    xp[:, padding:padding + length] = x
    cols = np.stack([xp[:, kk: kk + stride * (out_len - 1) + 1: stride] for kk in range(k)], axis=1)
    # cols [IC][K][L_out] -> [IC*K][L_out] matches w.reshape(OC, IC*K)
    y = w.reshape(oc, ic * k).astype(F32) @ cols.reshape(ic * k, out_len)
    return (y + b[:, None]).astype(F32)


def conv_transpose1d(x, w, b, stride=2, padding=1):
    """x [IC][L] -> [OC][L*stride]; weight [IC][OC][K] (diffusion_ops.cc:177-282).

    Output index ot = it*stride + k - padding."""
    ic, oc, k = w.shape
    length = x.shape[1]
    out_len = length * stride
    y = np.tile(b[:, None], (1, out_len)).astype(F32)
    for kk in range(k):
        contrib = w[:, :, kk].T.astype(F32) @ x  # [OC][L]
        for it in range(length):
            ot = it * stride + kk - padding
            if 0 <= ot < out_len:
                y[:, ot] += contrib[:, it]
    return y.astype(F32)


def group_norm(x, weight, bias, groups, eps=1e-5):
    """GroupNorm with float64 statistics, biased variance E[x^2]-E[x]^2 clamped at 0
    (diffusion_ops.cc:284-365)."""
    channels, length = x.shape
    xg = x.reshape(groups, (channels // groups) * length).astype(np.float64)
    mean = xg.mean(axis=1)
    var = np.maximum(0.0, (xg * xg).mean(axis=1) - mean * mean)
    inv = (1.0 / np.sqrt(var + eps)).astype(F32)
    mean_f = mean.astype(F32)
    cpg = channels // groups
    out = np.empty_like(x, dtype=F32)
    for g in range(groups):
        sl = slice(g * cpg, (g + 1) * cpg)
        scale = (inv[g] * weight[sl]).astype(F32)
        out[sl] = (x[sl] - mean_f[g]) * scale[:, None] + bias[sl][:, None]
    return out.astype(F32)


def timestep_embedding(timestep, dim):
    """[sin | cos](t * exp(-ln(1e4)/(half-1) * i)) (diffusion_ops.cc:379-396)."""
    half = dim // 2
    factor = F32(math.log(10000.0)) / F32(half - 1)
    freq = np.exp(-factor * np.arange(half, dtype=F32)).astype(F32)
    phase = (F32(timestep) * freq).astype(F32)
    return np.concatenate([np.sin(phase), np.cos(phase)]).astype(F32)


def alphas_cumprod(train_timesteps):
    """squaredcos_cap_v2: beta in float64, cumulative product in float32
    (diffusion.cc:186-191, 529-541)."""

    def alpha_bar(t):
        c = math.cos(((t + 0.008) / 1.008) * (math.pi / 2.0))
        return c * c

    out = np.empty(train_timesteps, F32)
    cumulative = F32(1)
    for step in range(train_timesteps):
        beta = F32(min(1.0 - alpha_bar((step + 1) / train_timesteps) / alpha_bar(step / train_timesteps), 0.999))
        cumulative = F32(cumulative * (F32(1) - beta))
        out[step] = cumulative
    return out


class GaussianGenerator:
    """splitmix64 -> 24-bit uniform -> Box-Muller, cos first (diffusion.cc:193-231).

    `uniform` divides in float32 by float(16777217) == 16777216, exactly as the
    C++ expression `static_cast<float>(...) / 16777217.0F` does."""

    MASK = 0xFFFFFFFFFFFFFFFF
    GOLDEN = 0x9E3779B97F4A7C15

    def __init__(self, seed):
        self.state = (int(seed) + self.GOLDEN) & self.MASK
        self.spare = F32(0)
        self.has_spare = False

    def _integer(self):
        self.state = (self.state + self.GOLDEN) & self.MASK
        v = self.state
        v = ((v ^ (v >> 30)) * 0xBF58476D1CE4E5B9) & self.MASK
        v = ((v ^ (v >> 27)) * 0x94D049BB133111EB) & self.MASK
        return v ^ (v >> 31)

    def _uniform(self):
        return F32(F32((self._integer() >> 40) + 1) / F32(16777217.0))

    def next(self):
        if self.has_spare:
            self.has_spare = False
            return self.spare
        first = max(self._uniform(), np.finfo(F32).tiny)
        second = self._uniform()
        radius = np.sqrt(F32(-2.0) * np.log(F32(first)), dtype=F32)
        angle = F32(F32(2.0 * math.pi) * second)
        self.spare = F32(radius * np.sin(angle, dtype=F32))
        self.has_spare = True
        return F32(radius * np.cos(angle, dtype=F32))

    def fill(self, n):
        return np.array([self.next() for _ in range(n)], F32)


class DiffusionModel:
    """LeRobot ConditionalUnet1D as loaded by DiffusionHead (diffusion.cc:383-541)."""

    def __init__(self, tensors):
        t = {k: np.asarray(v, F32) for k, v in tensors.items()}
        self.t = t
        meta = t["dp.meta"]
        self.action_dim = int(meta[1])
        self.horizon = int(meta[2])
        self.condition_dim = int(meta[5])
        self.stages = int(meta[6])
        self.kernel = int(meta[7])
        self.groups = int(meta[8])
        self.timestep_dim = int(meta[9])
        self.train_timesteps = int(meta[10])
        self.clip_sample = bool(int(meta[13]))
        self.clip_range = F32(meta[14])
        self.dims = [int(v) for v in t["dp.dims"]]
        self.action_min = t["dp.action_min"]
        self.action_max = t["dp.action_max"]
        self.alphas = alphas_cumprod(self.train_timesteps)

    def _residual(self, x, prefix, features):
        """diffusion.cc:724-773: conv1 -> GN -> Mish -> FiLM -> conv2 -> GN -> Mish -> +res."""
        t = self.t
        h = conv1d(x, t[prefix + ".c1.w"], t[prefix + ".c1.b"])
        h = mish(group_norm(h, t[prefix + ".n1.w"], t[prefix + ".n1.b"], self.groups))
        mod = (t[prefix + ".film.w"] @ features + t[prefix + ".film.b"]).astype(F32)
        oc = h.shape[0]
        h = (mod[:oc, None] * h + mod[oc:, None]).astype(F32)
        h = conv1d(h, t[prefix + ".c2.w"], t[prefix + ".c2.b"])
        h = mish(group_norm(h, t[prefix + ".n2.w"], t[prefix + ".n2.b"], self.groups))
        if prefix + ".res.w" in t:
            res = conv1d(x, t[prefix + ".res.w"], t[prefix + ".res.b"], padding=0)
        else:
            res = x
        return (h + res).astype(F32)

    def features(self, condition, timestep):
        """mish([time MLP(sinusoid(t)) | condition]) (diffusion.cc:806-820)."""
        t = self.t
        raw = timestep_embedding(timestep, self.timestep_dim)
        hidden = mish(t["dp.te1.w"] @ raw + t["dp.te1.b"])
        temb = (t["dp.te2.w"] @ hidden + t["dp.te2.b"]).astype(F32)
        return mish(np.concatenate([temb, np.asarray(condition, F32)]))

    def denoise(self, condition, sample, timestep):
        """Epsilon prediction, [H][A] in and out (diffusion.cc:793-914)."""
        t = self.t
        feats = self.features(condition, timestep)
        x = np.asarray(sample, F32).T.copy()  # [A][H]
        skips = []
        for stage in range(self.stages):
            for block in range(2):
                x = self._residual(x, f"dp.d{stage}.r{block}", feats)
            skips.append(x)
            if stage + 1 < self.stages:
                x = conv1d(x, t[f"dp.d{stage}.ds.w"], t[f"dp.d{stage}.ds.b"], stride=2, padding=1)
        for block in range(2):
            x = self._residual(x, f"dp.m{block}", feats)
        for stage in range(self.stages - 1):
            x = np.concatenate([x, skips[self.stages - 1 - stage]], axis=0)
            for block in range(2):
                x = self._residual(x, f"dp.u{stage}.r{block}", feats)
            x = conv_transpose1d(x, t[f"dp.u{stage}.us.w"], t[f"dp.u{stage}.us.b"])
        x = conv1d(x, t["dp.f.c.w"], t["dp.f.c.b"])
        x = mish(group_norm(x, t["dp.f.n.w"], t["dp.f.n.b"], 8))
        x = conv1d(x, t["dp.f.o.w"], t["dp.f.o.b"], padding=0)
        return x.T.copy()

    def schedule(self, steps):
        """timestep_i = (S-1-i) * (T // S); previous = timestep - ratio (diffusion.cc:984-990)."""
        ratio = self.train_timesteps // steps
        return [((steps - 1 - i) * ratio, (steps - 1 - i) * ratio - ratio) for i in range(steps)]

    def sample(self, condition, noise, steps, scheduler="ddim", seed=0, return_normalized=False):
        """DDIM (eta 0) / DDPM loop + MIN_MAX unnormalize (diffusion.cc:979-1034)."""
        x = np.asarray(noise, F32).copy()
        gaussian = GaussianGenerator(seed)
        for timestep, previous in self.schedule(steps):
            eps = self.denoise(condition, x, float(timestep))
            x = self.update(x, eps, timestep, previous, scheduler, gaussian)
        if return_normalized:
            return x
        return self.unnormalize(x)

    def update(self, x, eps, timestep, previous, scheduler, gaussian=None):
        """One scheduler update (diffusion.cc:997-1024)."""
        alpha_t = self.alphas[timestep]
        alpha_prev = self.alphas[previous] if previous >= 0 else F32(1)
        beta_t = F32(1) - alpha_t
        pred = ((x - np.sqrt(beta_t) * eps) / np.sqrt(alpha_t)).astype(F32)
        if self.clip_sample:
            pred = np.clip(pred, -self.clip_range, self.clip_range)
        if scheduler == "ddim":
            return (np.sqrt(alpha_prev) * pred + np.sqrt(F32(1) - alpha_prev) * eps).astype(F32)
        current_alpha = F32(alpha_t / alpha_prev)
        current_beta = F32(1) - current_alpha
        denom = max(beta_t, F32(1e-20))
        orig_coef = F32(np.sqrt(alpha_prev) * current_beta / denom)
        sample_coef = F32(np.sqrt(current_alpha) * (F32(1) - alpha_prev) / denom)
        variance = F32((F32(1) - alpha_prev) / denom * current_beta)
        nxt = (orig_coef * pred + sample_coef * x).astype(F32)
        if previous >= 0:
            noise = gaussian.fill(x.size).reshape(x.shape)
            nxt = (nxt + np.sqrt(max(variance, F32(1e-20))) * noise).astype(F32)
        return nxt

    def unnormalize(self, x):
        return ((x + F32(1)) * F32(0.5) * (self.action_max - self.action_min) + self.action_min).astype(F32)


# --------------------------------------------------------------------------
# flow-matching head (src/core/heads/flow/flow.cc)


class FlowModel:
    """Velocity MLP and resumable ODE sampler (flow.cc:64-323)."""

    def __init__(self, tensors):
        t = {k: np.asarray(v, F32) for k, v in tensors.items() if k.startswith("flow.")}
        self.w_in = t["flow.in_proj.weight"]
        self.w_time = t["flow.time_proj.weight"]
        self.w_cond = t["flow.cond_proj.weight"]
        self.w_out = t["flow.out_proj.weight"]
        self.layers = []
        while f"flow.layers.{len(self.layers)}.weight" in t:
            self.layers.append(t[f"flow.layers.{len(self.layers)}.weight"])
        self.action_dim = self.w_in.shape[1]
        self.hidden = self.w_in.shape[0]
        half = self.w_time.shape[1] // 2
        # flow.cc:104: f_j = 10000^(-j/half) in float32 pow.
        self.freqs = np.array([np.power(F32(10000.0), F32(-F32(j) / F32(half)), dtype=F32)
                               for j in range(half)], F32)

    def velocity(self, x, t, c_emb):
        """flow.cc:152-184; x may be [A] or [B][A] (rows independent)."""
        x = np.asarray(x, F32)
        phase = (F32(t) * self.freqs).astype(F32)
        sinu = np.concatenate([np.sin(phase), np.cos(phase)]).astype(F32)
        h = x @ self.w_in.T + (self.w_time @ sinu) + c_emb
        h = silu(h)
        for w in self.layers:
            h = silu(h @ w.T)
        return (h @ self.w_out.T).astype(F32)

    def sample(self, condition, x0, steps, solver="euler"):
        """flow.cc:210-323 (Euler / Heun / classic RK4, t_i = i/S)."""
        c_emb = (np.asarray(condition, F32) @ self.w_cond.T).astype(F32)
        x = np.asarray(x0, F32).copy()
        dt = F32(1) / F32(steps)
        for i in range(steps):
            t = F32(i) * dt
            k1 = self.velocity(x, t, c_emb)
            if solver == "euler":
                x = (x + dt * k1).astype(F32)
            elif solver == "heun":
                probe = (x + dt * k1).astype(F32)
                k2 = self.velocity(probe, t + dt, c_emb)
                x = (x + F32(0.5) * dt * (k1 + k2)).astype(F32)
            else:
                half = F32(0.5) * dt
                k2 = self.velocity((x + half * k1).astype(F32), t + half, c_emb)
                k3 = self.velocity((x + half * k2).astype(F32), t + half, c_emb)
                k4 = self.velocity((x + dt * k3).astype(F32), t + dt, c_emb)
                x = (x + dt / F32(6) * (k1 + F32(2) * k2 + F32(2) * k3 + k4)).astype(F32)
        return x


# --------------------------------------------------------------------------
# Mamba encoder (src/core/models/mamba/mamba.cc)


def selective_scan(delta, a_neg, b, u, c, d_skip, h=None):
    """h = exp(dt*A)h + dt*B*u; y = D*u + sum_n h*C (kernels_scalar.cc:133-169).

    delta, u: [L][di]; b, c: [L][ds]; a_neg: [ds][di]; returns (y, h)."""
    length, di = u.shape
    ds = a_neg.shape[0]
    h = np.zeros((ds, di), F32) if h is None else h.astype(F32).copy()
    y = np.empty((length, di), F32)
    for t in range(length):
        da = np.exp(delta[t][None, :] * a_neg).astype(F32)
        dbu = (delta[t][None, :] * b[t][:, None] * u[t][None, :]).astype(F32)
        h = (da * h + dbu).astype(F32)
        y[t] = d_skip * u[t] + np.sum(h * c[t][:, None], axis=0, dtype=F32)
    return y.astype(F32), h


class MambaModel:
    """Mamba prefill / decode (mamba.cc:103-382)."""

    def __init__(self, tensors):
        t = {k: np.asarray(v, F32) for k, v in tensors.items() if k.startswith("backbone.")}
        self.t = t
        self.embedding = t["backbone.embeddings.weight"]
        self.d_model = self.embedding.shape[1]
        a0 = t["backbone.layers.0.mixer.A_log"]
        self.d_inner, self.d_state = a0.shape
        self.d_conv = t["backbone.layers.0.mixer.conv1d.weight"].shape[2]
        self.dt_rank = t["backbone.layers.0.mixer.x_proj.weight"].shape[0] - 2 * self.d_state
        self.n_layers = 0
        while f"backbone.layers.{self.n_layers}.norm.weight" in t:
            self.n_layers += 1

    def _layer(self, i):
        p = f"backbone.layers.{i}."
        t = self.t
        return dict(norm=t[p + "norm.weight"], in_proj=t[p + "mixer.in_proj.weight"],
                    conv_w=t[p + "mixer.conv1d.weight"][:, 0, :], conv_b=t[p + "mixer.conv1d.bias"],
                    x_proj=t[p + "mixer.x_proj.weight"], dt_w=t[p + "mixer.dt_proj.weight"],
                    dt_b=t[p + "mixer.dt_proj.bias"],
                    a_neg=(-np.exp(t[p + "mixer.A_log"])).T.astype(F32).copy(),
                    d=t[p + "mixer.D"], out_proj=t[p + "mixer.out_proj.weight"])

    def layer_forward(self, lw, hidden):
        """mamba.cc:232-301."""
        di, ds, dr, dc = self.d_inner, self.d_state, self.dt_rank, self.d_conv
        length = hidden.shape[0]
        normed = rmsnorm(hidden, lw["norm"])
        xz = (normed @ lw["in_proj"].T).astype(F32)
        x, z = xz[:, :di], xz[:, di:]
        conv = np.tile(lw["conv_b"][None, :], (length, 1)).astype(F32)
        for k in range(dc):
            start = dc - 1 - k
            conv[start:] += lw["conv_w"][:, k][None, :] * x[: length - start]
        u = silu(conv)
        dbl = (u @ lw["x_proj"].T).astype(F32)
        dt = softplus(dbl[:, :dr] @ lw["dt_w"].T + lw["dt_b"])
        y, _ = selective_scan(dt, lw["a_neg"], dbl[:, dr:dr + ds], u, dbl[:, dr + ds:], lw["d"])
        y = (y * silu(z)).astype(F32)
        return (hidden + y @ lw["out_proj"].T).astype(F32)

    def forward_embeddings(self, hidden):
        """mamba.cc:303-315 (final RMSNorm after all layers)."""
        hidden = np.asarray(hidden, F32).copy()
        for i in range(self.n_layers):
            hidden = self.layer_forward(self._layer(i), hidden)
        return rmsnorm(hidden, self.t["backbone.norm_f.weight"])

    def run(self, tokens):
        """fe_engine_run: embedding rows then forward (engine_runtime.cc:595-635)."""
        return self.forward_embeddings(self.embedding[np.asarray(tokens)])

    def state_size(self):
        return self.n_layers * self.d_inner * (self.d_conv + self.d_state)

    def decode(self, token, state):
        """Streaming one-token step; state [layers][di*(dc+ds)] (mamba.cc:317-382)."""
        di, ds, dr, dc = self.d_inner, self.d_state, self.dt_rank, self.d_conv
        hidden = self.embedding[int(token)].astype(F32).copy()
        per = di * (dc + ds)
        for i in range(self.n_layers):
            lw = self._layer(i)
            window = state[i * per: i * per + di * dc].reshape(di, dc)
            h = state[i * per + di * dc: (i + 1) * per].reshape(ds, di)
            normed = rmsnorm(hidden[None, :], lw["norm"])[0]
            xz = (lw["in_proj"] @ normed).astype(F32)
            window[:, :-1] = window[:, 1:].copy()
            window[:, -1] = xz[:di]
            u = silu(np.sum(lw["conv_w"] * window, axis=1, dtype=F32) + lw["conv_b"])
            dbl = (lw["x_proj"] @ u).astype(F32)
            dt = softplus(lw["dt_w"] @ dbl[:dr] + lw["dt_b"])
            y, hn = selective_scan(dt[None, :], lw["a_neg"], dbl[None, dr:dr + ds], u[None, :],
                                   dbl[None, dr + ds:], lw["d"], h)
            h[:] = hn
            y = (y[0] * silu(xz[di:])).astype(F32)
            hidden = (hidden + lw["out_proj"] @ y).astype(F32)
        return rmsnorm(hidden[None, :], self.t["backbone.norm_f.weight"])[0]


# --------------------------------------------------------------------------
# SmolVLA flow action expert (src/core/models/smolvla/smolvla_action_expert.cc)


def round_bf16(x):
    """round_to_bf16 (src/core/kernels/kernels.h:236-244): round to nearest
    even in the bit pattern, no NaN special case."""
    bits = np.ascontiguousarray(x, F32).view(np.uint32)
    bias = ((bits >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    return ((bits + bias) & np.uint32(0xFFFF0000)).view(F32)


def rmsnorm_bf16(x, weight, eps=1e-5):
    """kernels.h:246-265: scale in f32, bf16 after the scale and after the weight."""
    x = np.asarray(x, F32)
    ss = np.sum(x * x, axis=-1, dtype=F32, keepdims=True)
    scale = (F32(1) / np.sqrt(ss / F32(x.shape[-1]) + F32(eps))).astype(F32)
    return round_bf16(round_bf16(x * scale) * np.asarray(weight, F32))


def apply_rope(x, head_width, position_base):
    """Interleaved-halves RoPE on [rows][heads][head_width] (kernels.h:339-362)."""
    half = head_width // 2
    c = np.arange(half, dtype=F32)
    exponent = ((F32(2) * c) / F32(head_width)).astype(F32)
    denom = np.exp(F32(9.210340371976184) * exponent).astype(F32)
    pos = (F32(position_base) + np.arange(x.shape[0], dtype=F32)).astype(F32)
    angle = (pos[:, None] / denom[None, :]).astype(F32)
    sin, cos = np.sin(angle)[:, None, :], np.cos(angle)[:, None, :]
    first, second = x[..., :half], x[..., half:]
    out = np.empty_like(x)
    out[..., :half] = first * cos - second * sin
    out[..., half:] = second * cos + first * sin
    return out.astype(F32)


def softmax_rows(s):
    """kernels.h:181-194 per row: exp(s - max), then times 1 / sum."""
    m = np.max(s, axis=-1, keepdims=True)
    e = np.exp((s - m).astype(F32)).astype(F32)
    inv = (F32(1) / np.sum(e, axis=-1, dtype=F32, keepdims=True)).astype(F32)
    return (e * inv).astype(F32)


class SmolVLAExpert:
    """Parameterised restatement of SmolVLAActionExpert (smolvla_action_expert.cc:209-477).

    The reference fixes the head width at 64 with 15 query and 5 K / V heads
    (:120-128); here they come from the checkpoint (`flowedge.smolvla.head_width`,
    default 64).  Cross-attention layers (odd) project the per-layer prefix
    cache; self-attention layers (even) attend over [cache ; action tokens]
    when the cache width equals the K / V width (the reference's layout), else
    over the action tokens only.  All bf16 rounding points are the reference's.
    """

    PREFIX = "model.vlm_with_expert.lm_expert."

    def __init__(self, tensors):
        t = {k: np.asarray(v, F32) for k, v in tensors.items()}
        self.w_in, self.b_in = t["model.action_in_proj.weight"], t["model.action_in_proj.bias"]
        self.w_out, self.b_out = t["model.action_out_proj.weight"], t["model.action_out_proj.bias"]
        self.w_tin, self.b_tin = t["model.action_time_mlp_in.weight"], t["model.action_time_mlp_in.bias"]
        self.w_tout, self.b_tout = t["model.action_time_mlp_out.weight"], t["model.action_time_mlp_out.bias"]
        self.final_norm = t[self.PREFIX + "norm.weight"]
        self.width = self.w_in.shape[0]
        self.action_dim = self.w_in.shape[1]
        hw = t.get("flowedge.smolvla.head_width")
        self.head_width = int(hw[0]) if hw is not None else 64
        self.layers = []
        while self.PREFIX + f"layers.{len(self.layers)}.self_attn.q_proj.weight" in t:
            p = self.PREFIX + f"layers.{len(self.layers)}."
            self.layers.append({k: t[p + k] for k in (
                "input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_proj.weight",
                "self_attn.k_proj.weight", "self_attn.v_proj.weight", "self_attn.o_proj.weight",
                "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight")})
        self.heads = self.layers[0]["self_attn.q_proj.weight"].shape[0] // self.head_width
        self.kv_heads = self.layers[0]["self_attn.k_proj.weight"].shape[0] // self.head_width
        self.kv_width = self.kv_heads * self.head_width
        self.cache_width = (self.layers[1]["self_attn.k_proj.weight"].shape[1] if len(self.layers) > 1
                            else self.kv_width)

    def embed_suffix(self, noisy, timestep):
        """smolvla_action_expert.cc:209-256."""
        noisy = np.asarray(noisy, F32).reshape(-1, self.action_dim)
        action = (noisy @ self.w_in.T + self.b_in).astype(F32)
        half = self.width // 2
        i = np.arange(half, dtype=F32)
        fraction = (i / F32(half - 1)).astype(F32)
        period = (F32(0.004) * np.power(F32(4.0) / F32(0.004), fraction).astype(F32)).astype(F32)
        angle = ((F32(2.0) * F32(3.14159265358979323846) / period) * F32(timestep)).astype(F32)
        time = np.concatenate([np.sin(angle), np.cos(angle)]).astype(F32)
        fused = np.concatenate([action, np.broadcast_to(time, action.shape)], axis=1)
        h = silu((fused @ self.w_tin.T).astype(F32) + self.b_tin)
        return ((h @ self.w_tout.T).astype(F32) + self.b_tout).astype(F32)

    def _attention(self, q, k, v, prefix_k, prefix_v, mask, cross):
        """grouped_query_attention (kernels.h:275-336) on [rows][heads][hw]."""
        rows, hw = q.shape[0], self.head_width
        groups = self.heads // self.kv_heads
        scale = F32(np.sqrt(F32(hw)))
        out = np.zeros((rows, self.heads, hw), F32)
        valid = mask.astype(bool)
        causal = np.tril(np.ones((rows, rows), bool))
        for h in range(self.heads):
            kh = h // groups
            parts, vals = [], []
            if cross:
                s = ((q[:, h, :] @ k[:, kh, :].T).astype(F32) / scale).astype(F32)
                s[:, ~valid] = -np.inf
                parts.append(s)
                vals.append(v[:, kh, :])
            else:
                if prefix_k is not None:
                    s = ((q[:, h, :] @ prefix_k[:, kh, :].T).astype(F32) / scale).astype(F32)
                    s[:, ~valid] = -np.inf
                    parts.append(s)
                    vals.append(prefix_v[:, kh, :])
                s = ((q[:, h, :] @ k[:, kh, :].T).astype(F32) / scale).astype(F32)
                s[~causal] = -np.inf
                parts.append(s)
                vals.append(v[:, kh, :])
            p = round_bf16(softmax_rows(np.concatenate(parts, axis=1)))
            out[:, h, :] = p @ np.concatenate(vals, axis=0)
        return out.reshape(rows, self.heads * hw)

    def run(self, suffix, keys, values, mask):
        """run_with_prefix_kv (smolvla_action_expert.cc:277-394); keys / values
        [layers][prefix][cache_width], mask [prefix]."""
        out = np.asarray(suffix, F32).reshape(-1, self.width).copy()
        rows, hw = out.shape[0], self.head_width
        mask = np.asarray(mask, np.uint8)
        valid = int(mask.sum())
        for li, L in enumerate(self.layers):
            cross = li % 2 == 1
            normed = round_bf16(rmsnorm_bf16(out, L["input_layernorm.weight"]))
            q = round_bf16(normed @ L["self_attn.q_proj.weight"].T).reshape(rows, self.heads, hw)
            prefix_k = prefix_v = None
            if cross:
                k = round_bf16(keys[li] @ L["self_attn.k_proj.weight"].T).reshape(-1, self.kv_heads, hw)
                v = round_bf16(values[li] @ L["self_attn.v_proj.weight"].T).reshape(-1, self.kv_heads, hw)
                q = apply_rope(q, hw, 0)
            else:
                k = round_bf16(normed @ L["self_attn.k_proj.weight"].T).reshape(rows, self.kv_heads, hw)
                v = round_bf16(normed @ L["self_attn.v_proj.weight"].T).reshape(rows, self.kv_heads, hw)
                q = apply_rope(q, hw, valid)
                k = round_bf16(apply_rope(k, hw, valid))
                if self.cache_width == self.kv_width:
                    prefix_k = np.asarray(keys[li], F32).reshape(-1, self.kv_heads, hw)
                    prefix_v = np.asarray(values[li], F32).reshape(-1, self.kv_heads, hw)
            q = round_bf16(q)
            att = round_bf16(self._attention(q, k, v, prefix_k, prefix_v, mask, cross))
            proj = round_bf16(att @ L["self_attn.o_proj.weight"].T)
            out = round_bf16(out + proj)
            normed = round_bf16(rmsnorm_bf16(out, L["post_attention_layernorm.weight"]))
            gate = round_bf16(normed @ L["mlp.gate_proj.weight"].T)
            up = round_bf16(normed @ L["mlp.up_proj.weight"].T)
            gate = round_bf16(up * silu(gate))
            proj = round_bf16(gate @ L["mlp.down_proj.weight"].T)
            out = round_bf16(out + proj)
        return round_bf16(rmsnorm_bf16(out, self.final_norm))

    def project_actions(self, hidden):
        """smolvla_action_expert.cc:258-275."""
        hidden = np.asarray(hidden, F32).reshape(-1, self.width)
        return ((hidden @ self.w_out.T).astype(F32) + self.b_out).astype(F32)

    def denoise(self, noisy, timestep, keys, values, mask):
        """denoise_with_prefix_kv (smolvla_action_expert.cc:396-420)."""
        hidden = self.run(self.embed_suffix(noisy, timestep), keys, values, mask)
        return self.project_actions(hidden)

    def sample(self, noise, steps, keys, values, mask):
        """sample_euler_with_prefix_kv (smolvla_action_expert.cc:422-474):
        t = 1 + step * dt, dt = -1 / steps; noise [chunk][action_dim]."""
        x = np.asarray(noise, F32).reshape(-1, self.action_dim).copy()
        dt = F32(-1.0) / F32(steps)
        for step in range(steps):
            t = F32(F32(1.0) + F32(step) * dt)
            v = self.denoise(x, t, keys, values, mask)
            x = (x + dt * v).astype(F32)
        return x
