"""Per-model declarations as data: defaults, guidance kind, refusals, prompt budgets.

The CLI, the serving validator and the applications read one ``ModelSpec`` per model
instead of each carrying its own copy of the same checks (the reference's spec-as-data
pattern, difflet/models/spec.py:33-78, per-model specs difflet/models/*/spec.py).  This
module imports no torch: a serving parent process reads specs without loading it.

The refusals here are this engine's own: every parallel mode is native on B200, TeaCache
runs for the MMDiT family and Wan, and bucketed request shapes are supported by the
compile cache, so fewer options are refused than in the reference's GPU flow.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class PromptBudget:
    """One text encoder's token limit, as the serving validator checks it."""

    encoder: str
    max_tokens: int
    #: message for a prompt over the limit; ``{name}`` is ``prompt`` or ``negative_prompt``
    too_long: str
    applies_to_negative_prompt: bool = False


@dataclass(frozen=True)
class ModelSpec:
    model_type: str
    display_name: str
    short_name: str
    #: checkpoints ``difflet run`` routes to this model (the first is the default)
    cli_model_ids: tuple
    #: checkpoints ``difflet serve`` accepts
    served_checkpoint_ids: tuple
    output: str  # "image" | "video"
    default_height: int
    default_width: int
    default_num_frames: int | None
    default_steps: int
    #: "none": no guidance input; "distilled": one pass with the scale as an input;
    #: "cfg": two branches per step (batched, or split over the cfg axis)
    guidance: str
    default_guidance_scale: float | None
    max_guidance_scale: float = 20.0
    default_fps: int | None = None
    accepts_negative_prompt: bool = False
    #: CLI options the model refuses: (argparse attribute, how the message names it)
    refused_cli_flags: tuple = ()
    #: video request fields the model refuses: (field, why)
    refused_video_fields: tuple = ()
    #: generate() keyword arguments the model refuses when they carry a value
    refused_generate_kwargs: tuple = ()
    refused_reason: str = ""
    prompt_budgets: tuple = ()
    smoke_steps: int = 4
    smoke_prompt: str = "a small red square"
    #: "module:function" creating the application (imported only where torch is loaded)
    application: str = ""

    @property
    def accepts_cfg_parallel(self) -> bool:
        return self.guidance == "cfg"

    @property
    def takes_guidance_scale(self) -> bool:
        return self.guidance != "none"


_WAN_ONLY = ("guidance_scale_2", "--guidance-scale-2 (Wan's low-noise expert scale)")
_NO_TRUE_CFG = ("true_cfg_scale", "--true-cfg-scale (the model runs without a true-CFG branch)")

SPECS: dict[str, ModelSpec] = {
    "flux": ModelSpec(
        model_type="flux", display_name="FLUX.1", short_name="flux",
        cli_model_ids=("black-forest-labs/FLUX.1-dev", "black-forest-labs/FLUX.1-schnell"),
        served_checkpoint_ids=("black-forest-labs/FLUX.1-dev", "black-forest-labs/FLUX.1-schnell"),
        output="image", default_height=1024, default_width=1024, default_num_frames=None, default_steps=28,
        guidance="distilled", default_guidance_scale=3.5,
        refused_cli_flags=(_WAN_ONLY, _NO_TRUE_CFG, ("num_frames", "--num-frames (FLUX makes images)")),
        refused_generate_kwargs=("guidance_scale_2", "true_cfg_scale", "num_frames", "negative_prompt"),
        refused_reason="FLUX.1 is guidance-distilled: one branch, the scale is an input",
        prompt_budgets=(PromptBudget("t5", 512, "FLUX {name} exceeds T5's 512 tokens"),),
        application="difflet_b200.models.flux.entry:create_application"),
    "wan": ModelSpec(
        model_type="wan", display_name="Wan 2.2", short_name="wan",
        cli_model_ids=("Wan-AI/Wan2.2-T2V-A14B-Diffusers", "Wan-AI/Wan2.1-T2V-14B-Diffusers"),
        served_checkpoint_ids=("Wan-AI/Wan2.2-T2V-A14B-Diffusers",),
        output="video", default_height=720, default_width=1280, default_num_frames=81, default_steps=40,
        guidance="cfg", default_guidance_scale=4.0, default_fps=16, accepts_negative_prompt=True,
        refused_cli_flags=(_NO_TRUE_CFG,),
        refused_video_fields=(("true_cfg_scale", "Wan already runs true CFG; use guidance_scale / guidance_scale_2"),),
        refused_generate_kwargs=("true_cfg_scale",),
        refused_reason="Wan's CFG scales are guidance_scale (high-noise expert) and guidance_scale_2",
        prompt_budgets=(PromptBudget("umt5", 512, "Wan {name} exceeds UMT5's 512 tokens",
                                     applies_to_negative_prompt=True),),
        application="difflet_b200.models.wan.entry:create_application"),
    "hunyuan_video": ModelSpec(
        model_type="hunyuan_video", display_name="HunyuanVideo", short_name="hunyuan",
        cli_model_ids=("hunyuanvideo-community/HunyuanVideo", "tencent/HunyuanVideo"),
        served_checkpoint_ids=("hunyuanvideo-community/HunyuanVideo",),
        output="video", default_height=720, default_width=1280, default_num_frames=129, default_steps=50,
        guidance="distilled", default_guidance_scale=6.0, default_fps=24, accepts_negative_prompt=True,
        refused_cli_flags=(_WAN_ONLY,),
        refused_generate_kwargs=("guidance_scale_2",),
        refused_reason="HunyuanVideo has one expert (guidance_scale_2 is Wan's); a negative prompt needs true_cfg_scale",
        prompt_budgets=(PromptBudget("llama", 256, "HunyuanVideo {name} exceeds the text encoder's 256 tokens"),),
        application="difflet_b200.models.hunyuan_video.entry:create_application"),
    "hunyuan_video_15": ModelSpec(
        model_type="hunyuan_video_15", display_name="HunyuanVideo 1.5", short_name="hv15",
        cli_model_ids=("hunyuanvideo-community/HunyuanVideo-1.5-Diffusers-480p_t2v",),
        served_checkpoint_ids=("hunyuanvideo-community/HunyuanVideo-1.5-Diffusers-480p_t2v",),
        output="video", default_height=480, default_width=848, default_num_frames=121, default_steps=50,
        guidance="cfg", default_guidance_scale=6.0, default_fps=24, accepts_negative_prompt=True,
        refused_cli_flags=(_WAN_ONLY,),
        refused_generate_kwargs=("guidance_scale_2",),
        refused_reason="HunyuanVideo 1.5 has one expert (guidance_scale_2 is Wan's)",
        prompt_budgets=(PromptBudget("qwen", 1000, "HunyuanVideo 1.5 {name} exceeds the text encoder's 1000 tokens",
                                     applies_to_negative_prompt=True),),
        application="difflet_b200.models.hunyuan_video.entry:create_application_15"),
    "qwen_image": ModelSpec(
        model_type="qwen_image", display_name="Qwen-Image", short_name="qwen",
        cli_model_ids=("Qwen/Qwen-Image",), served_checkpoint_ids=("Qwen/Qwen-Image",),
        output="image", default_height=1328, default_width=1328, default_num_frames=None, default_steps=50,
        guidance="cfg", default_guidance_scale=4.0, accepts_negative_prompt=True,
        refused_cli_flags=(_WAN_ONLY, ("num_frames", "--num-frames (Qwen-Image makes images)")),
        refused_generate_kwargs=("guidance_scale_2", "num_frames"),
        refused_reason="Qwen-Image is a single-expert image model",
        prompt_budgets=(PromptBudget("qwen2.5-vl", 1024, "Qwen-Image {name} exceeds the text encoder's 1024 tokens",
                                     applies_to_negative_prompt=True),),
        application="difflet_b200.models.qwen_image.entry:create_application"),
    "ltx_2": ModelSpec(
        model_type="ltx_2", display_name="LTX-2", short_name="ltx2",
        cli_model_ids=("Lightricks/LTX-2",), served_checkpoint_ids=("Lightricks/LTX-2",),
        output="video", default_height=512, default_width=768, default_num_frames=121, default_steps=40,
        guidance="cfg", default_guidance_scale=4.0, default_fps=24, accepts_negative_prompt=True,
        refused_cli_flags=(_WAN_ONLY, _NO_TRUE_CFG),
        refused_generate_kwargs=("guidance_scale_2", "true_cfg_scale"),
        refused_reason="LTX-2 guidance is guidance_scale / stg_scale / modality_scale",
        prompt_budgets=(PromptBudget("gemma-3", 1024, "LTX-2 {name} exceeds Gemma-3's 1024 tokens",
                                     applies_to_negative_prompt=True),),
        application="difflet_b200.models.ltx_2.entry:create_application"),
    "minimax_h3": ModelSpec(
        model_type="minimax_h3", display_name="MiniMax-H3", short_name="h3",
        cli_model_ids=("MiniMaxAI/MiniMax-H3",), served_checkpoint_ids=("MiniMaxAI/MiniMax-H3",),
        output="video", default_height=480, default_width=832, default_num_frames=124, default_steps=30,
        guidance="none", default_guidance_scale=None, default_fps=24,
        refused_cli_flags=(_WAN_ONLY, _NO_TRUE_CFG, ("guidance_scale", "--guidance-scale (MiniMax-H3 is guidance-free)"),
                           ("cfg_parallel", "--cfg-parallel (MiniMax-H3 runs one branch)")),
        refused_generate_kwargs=("guidance_scale", "guidance_scale_2", "true_cfg_scale", "negative_prompt"),
        refused_reason="MiniMax-H3 samples without classifier-free guidance",
        application="difflet_b200.models.minimax_h3.entry:create_application"),
}


class SpecRefusal(ValueError):
    """A request option the model does not take (message names the option and why)."""


def model_spec(model_type: str) -> ModelSpec | None:
    return SPECS.get(model_type)


def model_specs() -> tuple:
    return tuple(SPECS.values())


def spec_for_model_id(model_id: str) -> ModelSpec | None:
    """The spec whose CLI or served checkpoint ids list ``model_id``."""
    mid = model_id.rstrip("/")
    for spec in SPECS.values():
        if mid in spec.cli_model_ids or mid in spec.served_checkpoint_ids or mid == spec.model_type:
            return spec
    return None


def check_cli_args(spec: ModelSpec, args) -> None:
    """Refuse CLI options the model does not take (an argparse namespace; unset = None / False)."""
    bad = [name for attr, name in spec.refused_cli_flags if getattr(args, attr, None) not in (None, False, "", 0)]
    if bad:
        raise SpecRefusal(f"{spec.display_name} does not take {', '.join(bad)}")


def check_generate_kwargs(spec: ModelSpec, kwargs: dict) -> None:
    """Refuse generate() arguments the model does not take, and out-of-range guidance scales."""
    bad = [k for k in spec.refused_generate_kwargs if kwargs.get(k) not in (None, "", False)]
    if bad:
        raise SpecRefusal(f"{spec.display_name} does not take {', '.join(sorted(bad))}: {spec.refused_reason}")
    g = kwargs.get("guidance_scale")
    if g is not None and spec.takes_guidance_scale and not 0.0 <= float(g) <= spec.max_guidance_scale:
        raise SpecRefusal(f"guidance_scale must be in [0, {spec.max_guidance_scale}], got {g}")


def check_prompt_budgets(spec: ModelSpec, token_counts: dict) -> None:
    """``token_counts`` maps ``prompt`` / ``negative_prompt`` to {encoder: tokens}."""
    for name, counts in token_counts.items():
        for b in spec.prompt_budgets:
            if name == "negative_prompt" and not b.applies_to_negative_prompt:
                continue
            n = counts.get(b.encoder)
            if n is not None and n > b.max_tokens:
                raise SpecRefusal(b.too_long.format(name=name))


def generate_defaults(spec: ModelSpec) -> dict:
    """The generate() arguments a request without them gets."""
    d = {"height": spec.default_height, "width": spec.default_width, "num_inference_steps": spec.default_steps}
    if spec.default_num_frames is not None:
        d["num_frames"] = spec.default_num_frames
    if spec.default_guidance_scale is not None:
        d["guidance_scale"] = spec.default_guidance_scale
    return d


__all__ = ["ModelSpec", "PromptBudget", "SPECS", "SpecRefusal", "check_cli_args", "check_generate_kwargs",
           "check_prompt_budgets", "generate_defaults", "model_spec", "model_specs", "spec_for_model_id"]
