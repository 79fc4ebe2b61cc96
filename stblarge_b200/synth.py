"""Seeded synthetic MoE layers for tests and benchmarks (no checkpoints exist for this layer).

Weights are ~N(0, weight_std) floats quantized to the layer's formats by the same rules the
reference's torch stand-ins use (ref/kernel.py:35-45 applied to 128x128 blocks for FP8 weights,
ref/kernel.py:55-72 E8M0 branch for MXFP4).  Seeds: router W 1, bias 2, shared expert 3, x 4,
routed expert e 1000 + e.

Two generators:
  * host_layer(cfg): numpy PCG64 floats (exactly reproducible on any machine), quantized with torch on
    the CPU; used for the small configurations the CPU oracle checks, and by the golden fixtures.
  * device_layer(cfg, device): torch's CUDA generator, quantized on the GPU; used for the full-size
    layers (11 GB of FP8 experts), where host generation would take minutes.
"""

import numpy as np
import torch

from .config import FMT_FP8_B128, FMT_FP8_E8M0, FMT_MXFP4, FMT_NONE

FP4_GRID = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=torch.float32)


# ---- quantizers (torch, any device) -------------------------------------------------------------

def pow2_ceil(t):
    bits = t.float().contiguous().view(torch.int32)
    e = ((bits >> 23) & 0xFF) - 127 + ((bits & 0x7FFFFF) != 0).int()
    return ((e + 127) << 23).view(torch.float32)


def quant_fp8_b128(w):
    """float [rows, k] -> (e4m3 codes uint8 [rows, k], fp32 scales [ceil(rows/128), ceil(k/128)])."""
    rows, k = w.shape
    rb, kb = (rows + 127) // 128, (k + 127) // 128
    wp = torch.zeros(rb * 128, kb * 128, dtype=torch.float32, device=w.device)
    wp[:rows, :k] = w.float()
    blk = wp.view(rb, 128, kb, 128)
    amax = blk.abs().amax(dim=(1, 3)).clamp_min(1e-4)
    s = amax * torch.tensor(1.0 / 448.0, dtype=torch.float32, device=w.device)
    q = (blk / s[:, None, :, None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    codes = q.view(torch.uint8).view(rb * 128, kb * 128)[:rows, :k].contiguous()
    return codes, s.contiguous()


def quant_mxfp4(w):
    """float [rows, k] -> (packed e2m1 uint8 [rows, k/2], e8m0 scale bytes [rows, k/32])."""
    rows, k = w.shape
    b = w.float().reshape(rows, k // 32, 32)
    amax = b.abs().amax(-1).clamp_min(6.0 * 2.0 ** -126)
    s = pow2_ceil(amax * torch.tensor(1.0 / 6.0, dtype=torch.float32, device=w.device))
    v = (b / s.unsqueeze(-1)).clamp(-6.0, 6.0)
    a = v.abs()
    step = torch.where(a < 2, 0.5, torch.where(a < 4, 1.0, 2.0))
    q = torch.copysign(torch.round(a / step) * step, v)
    mag = torch.searchsorted(FP4_GRID.to(w.device), q.abs().contiguous())
    codes = (mag | (torch.signbit(q).int() << 3)).to(torch.uint8).view(rows, k // 2, 2)
    packed = (codes[..., 0] | (codes[..., 1] << 4)).contiguous()
    scales = ((s.view(torch.int32) >> 23) & 0xFF).to(torch.uint8).contiguous()
    return packed, scales


def quant_fp8_e8m0(w):
    """float [rows, k] -> (e4m3 codes uint8 [rows, k], e8m0 scale bytes [ceil(rows/32), k/32]): per 32x32
    block a power-of-two scale by act_quant's rule (amax clamp 1e-4, 2^ceil(log2(amax / 448)))."""
    rows, k = w.shape
    rb = (rows + 31) // 32
    wp = torch.zeros(rb * 32, k, dtype=torch.float32, device=w.device)
    wp[:rows] = w.float()
    blk = wp.view(rb, 32, k // 32, 32)
    amax = blk.abs().amax(dim=(1, 3)).clamp_min(1e-4)
    s = pow2_ceil(amax * torch.tensor(1.0 / 448.0, dtype=torch.float32, device=w.device))
    q = (blk / s[:, None, :, None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    codes = q.view(torch.uint8).view(rb * 32, k)[:rows].contiguous()
    scales = ((s.view(torch.int32) >> 23) & 0xFF).to(torch.uint8).contiguous()
    return codes, scales


def quantize(w, fmt):
    if fmt == FMT_FP8_B128:
        return quant_fp8_b128(w)
    if fmt == FMT_FP8_E8M0:
        return quant_fp8_e8m0(w)
    if fmt == FMT_MXFP4:
        return quant_mxfp4(w)
    raise ValueError(f"unknown weight format {fmt}")


# ---- activations ----------------------------------------------------------------------------------

def f32_to_bf16_bits(x):
    """numpy float32 -> bf16 bits, round to nearest even."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
    return b.astype(np.uint16)


def bf16_bits_to_f32(b):
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def make_x(hidden, T, seed=4):
    """T decode tokens, bf16 ~N(0, 1), as bf16 bits [T, hidden]."""
    return f32_to_bf16_bits(np.random.default_rng(seed).standard_normal((T, hidden), dtype=np.float32))


# ---- router ---------------------------------------------------------------------------------------

def router_bias(cfg):
    rng = np.random.default_rng(2)
    E = cfg.n_experts
    if cfg.zipf_s > 0:
        ranks = rng.permutation(E) + 1
        lnp = -cfg.zipf_s * np.log(ranks.astype(np.float64))
        return (cfg.zipf_c * (lnp - lnp.mean())).astype(np.float32)
    return (rng.standard_normal(E, dtype=np.float32) * np.float32(cfg.bias_std)).astype(np.float32)


def router_w(cfg):
    return (np.random.default_rng(1).standard_normal((cfg.n_experts, cfg.hidden), dtype=np.float32)
            * np.float32(cfg.router_std)).astype(np.float32)


# ---- host generator (small layers) ----------------------------------------------------------------

def expert_floats(cfg, seed):
    rng = np.random.default_rng(seed)
    H, I, sd = cfg.hidden, cfg.inter, np.float32(cfg.weight_std)
    gate = rng.standard_normal((I, H), dtype=np.float32) * sd
    up = rng.standard_normal((I, H), dtype=np.float32) * sd
    down = rng.standard_normal((H, I), dtype=np.float32) * sd
    return gate, up, down


def host_layer(cfg):
    """Quantized numpy weights: {'router_w', 'router_bias', 'routed': [m][e] -> (codes, scales),
    'shared': [m] -> (codes, scales) or None}."""
    routed = [[None] * cfg.n_experts for _ in range(3)]
    for e in range(cfg.n_experts):
        for m, w in enumerate(expert_floats(cfg, 1000 + e)):
            c, s = quantize(torch.from_numpy(w), cfg.routed_fmt)
            routed[m][e] = (c.numpy(), s.numpy())
    shared = None
    if cfg.shared_fmt != FMT_NONE:
        shared = []
        for w in expert_floats(cfg, 3):
            c, s = quantize(torch.from_numpy(w), cfg.shared_fmt)
            shared.append((c.numpy(), s.numpy()))
    return {"router_w": router_w(cfg), "router_bias": router_bias(cfg), "routed": routed, "shared": shared}


# ---- device generator (full-size layers) ----------------------------------------------------------

def _dev_floats(shape, seed, std, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.randn(*shape, generator=g, device=device, dtype=torch.float32) * std


def mat_shapes(cfg):
    H, I = cfg.hidden, cfg.inter
    return ((I, H), (I, H), (H, I))


def routed_expert(cfg, seed, device="cuda"):
    """One routed expert's quantized matrices (gate, up, down) and scales from seed `seed`."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    ws, ss = [], []
    for (r, k) in mat_shapes(cfg):
        w = torch.randn(r, k, generator=g, device=device, dtype=torch.float32) * cfg.weight_std
        c, s = quantize(w, cfg.routed_fmt)
        ws.append(c)
        ss.append(s)
    return ws, ss


def device_layer(cfg, device="cuda", experts=None, seed_base=1000):
    """Quantized device tensors in the expert-major layout the C ABI takes:
    'routed_w'[m]: uint8 [E, rows, codes per row]; 'routed_s'[m]: scales [E, ...];
    'shared_w'[m], 'shared_s'[m] likewise without the expert axis; 'router_w' fp32 [E, H];
    'router_bias' fp32 [E].  experts: the routed experts to build (a range: an expert-parallel
    rank's shard; expert e keeps seed seed_base + e), all by default."""
    experts = range(cfg.n_experts) if experts is None else experts
    E = len(experts)
    shapes = mat_shapes(cfg)
    routed_w, routed_s = [], []
    for m, (r, k) in enumerate(shapes):
        if cfg.routed_fmt == FMT_FP8_B128:
            routed_w.append(torch.empty(E, r, k, dtype=torch.uint8, device=device))
            routed_s.append(torch.empty(E, (r + 127) // 128, (k + 127) // 128, dtype=torch.float32, device=device))
        elif cfg.routed_fmt == FMT_FP8_E8M0:
            routed_w.append(torch.empty(E, r, k, dtype=torch.uint8, device=device))
            routed_s.append(torch.empty(E, (r + 31) // 32, k // 32, dtype=torch.uint8, device=device))
        else:
            routed_w.append(torch.empty(E, r, k // 2, dtype=torch.uint8, device=device))
            routed_s.append(torch.empty(E, r, k // 32, dtype=torch.uint8, device=device))
    for i, e in enumerate(experts):
        ws, ss = routed_expert(cfg, seed_base + e, device)
        for m in range(3):
            routed_w[m][i].copy_(ws[m])
            routed_s[m][i].copy_(ss[m])
    out = {"routed_w": routed_w, "routed_s": routed_s, "shared_w": None, "shared_s": None}
    if cfg.shared_fmt != FMT_NONE:
        g = torch.Generator(device=device)
        g.manual_seed(3)
        sw, ss = [], []
        for (r, k) in shapes:
            w = torch.randn(r, k, generator=g, device=device, dtype=torch.float32) * cfg.weight_std
            c, s = quantize(w, cfg.shared_fmt)
            sw.append(c)
            ss.append(s)
        out["shared_w"], out["shared_s"] = sw, ss
    out["router_w"] = torch.from_numpy(router_w(cfg)).to(device)
    out["router_bias"] = torch.from_numpy(router_bias(cfg)).to(device)
    return out


def device_to_host_expert(layer, e, m_count=3):
    """Copy routed expert e of a device layer to numpy [(codes, scales)] * 3 (for the oracle)."""
    return [(layer["routed_w"][m][e].cpu().numpy(), layer["routed_s"][m][e].cpu().numpy()) for m in range(m_count)]
