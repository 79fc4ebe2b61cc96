"""MoE layer configuration: shapes, routing rule and weight formats.

The presets are the layer configurations the B200 path is measured and checked on: a small layer
that the CPU oracle runs in seconds, and the full-size DeepSeek-V3-shaped layer (hidden 7168,
moe_intermediate 2048, 256 routed experts + 1 shared, top-8 over 8 groups keeping 4, sigmoid gate,
routed scaling 2.5) with FP8 128x128-block experts or MXFP4 experts.
"""

from dataclasses import asdict, dataclass, replace

# weight storage formats (ids shared with include/stbl_moe.h)
FMT_NONE = 0
FMT_FP8_B128 = 1  # e4m3 codes [rows][k], fp32 scales [ceil(rows/128)][ceil(k/128)]
FMT_MXFP4 = 2     # e2m1 codes [rows][k/2] (even index in the low nibble), e8m0 scales [rows][k/32]
FMT_FP8_E8M0 = 3  # e4m3 codes [rows][k], e8m0 scales [ceil(rows/32)][k/32]: the reference engine's FP8

# router score functions
SCORE_SIGMOID = 0          # DeepSeek-V3: sigmoid, group-limited top-k
SCORE_SQRT_SOFTPLUS = 1    # the reference engine (stbl/model.cu:430-431): sqrt(softplus)


@dataclass(frozen=True)
class MoEConfig:
    name: str
    hidden: int
    inter: int
    n_experts: int
    topk: int
    n_groups: int
    topk_groups: int
    score_fn: int = SCORE_SIGMOID
    route_scale: float = 2.5
    swiglu_limit: float = 0.0   # 0 disables the SwiGLU clamps (stbl/kernels.cu:457)
    routed_fmt: int = FMT_FP8_B128
    shared_fmt: int = FMT_FP8_B128
    weight_std: float = 0.02
    router_std: float = 0.02
    bias_std: float = 0.1
    zipf_s: float = 0.0         # > 0: correction bias skews expert popularity as Zipf(s)
    zipf_c: float = 0.5         # bias = zipf_c * (ln p_e - mean ln p)
    act_q8: int = 0             # 1: routed MXFP4 experts take Q8 activations (int8 per 32, scale amax/127)

    def as_dict(self):
        return asdict(self)

    def bytes_per_expert(self, fmt=None):
        """Stored bytes of one expert (gate + up + down, codes and scales)."""
        fmt = self.routed_fmt if fmt is None else fmt
        H, I = self.hidden, self.inter
        if fmt == FMT_FP8_B128:
            def mat(r, k):
                return r * k + 4 * ((r + 127) // 128) * ((k + 127) // 128)
        elif fmt == FMT_MXFP4:
            def mat(r, k):
                return r * k // 2 + r * (k // 32)
        elif fmt == FMT_FP8_E8M0:
            def mat(r, k):
                return r * k + ((r + 31) // 32) * (k // 32)
        else:
            return 0
        return 2 * mat(I, H) + mat(H, I)


CFG1 = MoEConfig("cfg1", hidden=1024, inter=512, n_experts=16, topk=4, n_groups=4, topk_groups=2)
CFG1_FP4 = replace(CFG1, name="cfg1_fp4", routed_fmt=FMT_MXFP4)
CFG2 = MoEConfig("cfg2", hidden=7168, inter=2048, n_experts=256, topk=8, n_groups=8, topk_groups=4)
CFG3 = replace(CFG2, name="cfg3", routed_fmt=FMT_MXFP4, zipf_s=1.0)
# the reference engine's own formats and routing: MXFP4 routed experts, FP8 shared expert with e8m0
# 32x32 block scales, per-32 power-of-two activation scales, sqrt(softplus) scores without group limit
CFG1_REF = replace(CFG1, name="cfg1_ref", routed_fmt=FMT_MXFP4, shared_fmt=FMT_FP8_E8M0, score_fn=SCORE_SQRT_SOFTPLUS,
                   n_groups=1, topk_groups=1)
CFG1_E8 = replace(CFG1, name="cfg1_e8", routed_fmt=FMT_FP8_E8M0, shared_fmt=FMT_FP8_E8M0)
CFG3_REF = replace(CFG2, name="cfg3_ref", routed_fmt=FMT_MXFP4, shared_fmt=FMT_FP8_E8M0, score_fn=SCORE_SQRT_SOFTPLUS,
                   n_groups=1, topk_groups=1)

# the Q8 activation variant of the MXFP4 layers (ref/emulate_ds4.py: routed MXFP4 experts take int8
# activations per 32 instead of FP8; the shared expert keeps FP8)
CFG1_Q8 = replace(CFG1_FP4, name="cfg1_q8", act_q8=1)
CFG3_Q8 = replace(CFG3, name="cfg3_q8", act_q8=1)

PRESETS = {c.name: c for c in (CFG1, CFG1_FP4, CFG2, CFG3, CFG1_REF, CFG1_E8, CFG3_REF, CFG1_Q8, CFG3_Q8)}
