"""The WEIGHTFERRY_* switches the quantized-weight path reads, with their defaults (core/env.py of the reference,
:16-135, restricted to the hot path's switches; same names, same precedence).

get(name) returns the environment variable if set, else the value from the settings file, else the default. The
settings file is ``WEIGHTFERRY_SETTINGS_FILE`` (a path; "0" / "off" / "" disables it) or, inside ComfyUI, the user
directory's ``weightferry.env``; lines ``NAME=value``, ``#`` starts a comment; read once per process. An unknown name
raises KeyError, so that a misspelt switch is an error rather than a silent default."""

import os

DEFAULTS = {
    "WEIGHTFERRY_GGUF_TRITON": "1",        # GGUF dequant through this package's kernels (name kept from the reference)
    "WEIGHTFERRY_GGUF_KQUANTS": "1",       # ... including the K-quants Q2_K .. Q6_K
    "WEIGHTFERRY_GGUF_LORA_FACTORS": "pin",  # LoRA factors of GGUF layers kept in pinned host memory
    "WEIGHTFERRY_FUSED_BLOCK": "1",        # fused Cosmos / Anima block parts: 1 / all / 0 / comma list
    "WEIGHTFERRY_CFG_RESID_MERGE": "1",    # one residual GEMM over all CFG rows when their gates are equal
    "WEIGHTFERRY_SLOTS": None,             # GPU slots of the block-streaming ring (None: the node's option)
    "WEIGHTFERRY_PREFETCH_PRIORITY": None,  # CUDA priority of the transfer stream (lower = higher)
    "WEIGHTFERRY_PROFILE": None,           # 1: CUDA-event timeline of the streaming pipeline
    "WEIGHTFERRY_AUTO": None,              # 1: the streaming node chooses resident blocks as with auto_config
    "WEIGHTFERRY_AUTO_HEADROOM_MB": "1536",  # VRAM auto_config leaves for activations
    "WEIGHTFERRY_VRAM_BUDGET_GB": None,    # most VRAM this process may use (the node's vram_budget_gb wins when > 0)
    "WEIGHTFERRY_TIERING": None,           # auto / ram: overrides the streaming node's tiering option
    "WEIGHTFERRY_RAM_BUDGET_GB": None,     # pinned-RAM budget of the streamed blocks (None: the node's option)
    "WEIGHTFERRY_RAM_MARGIN_GB": "6",      # RAM kept free when the budget is the available RAM
    "WEIGHTFERRY_DISK_DIR": None,          # folder of the SSD tier's cache files (None: ComfyUI's / the system temp)
    "WEIGHTFERRY_DISK_THREADS": None,      # SSD reader threads (None: the probe's fastest count)
    "WEIGHTFERRY_SSD_LAYOUT": "interleave",  # which streamed blocks go to the SSD: interleave / tail
    "WEIGHTFERRY_TP_CHUNKS": "1",          # row chunks of the tensor-parallel stack's overlapped sub-layers (1: off)
    "WEIGHTFERRY_SETTINGS_FILE": None,
}

_file = {"values": None}


def _settings_path():
    spec = os.environ.get("WEIGHTFERRY_SETTINGS_FILE")
    if spec is not None:
        return None if spec.strip().lower() in ("", "0", "off", "false", "none") else spec
    try:
        import folder_paths  # ComfyUI's
        return os.path.join(folder_paths.get_user_directory(), "weightferry.env")
    except Exception:  # noqa: BLE001 -- outside ComfyUI there is no default settings file
        return None


def file_values():
    """NAME -> value from the settings file (known names only); {} when there is none."""
    if _file["values"] is None:
        vals = {}
        path = _settings_path()
        lines = []
        if path:
            try:
                with open(path, encoding="utf-8") as f:
                    lines = f.read().splitlines()
            except OSError:
                lines = []
        for line in lines:
            s = line.strip()
            if not s or s.startswith("#") or "=" not in s:
                continue
            key, val = (x.strip() for x in s.split("=", 1))
            if key in DEFAULTS and key != "WEIGHTFERRY_SETTINGS_FILE":
                vals[key] = val
        _file["values"] = vals
    return _file["values"]


def reset_file_cache():
    _file["values"] = None


def get(name):
    default = DEFAULTS[name]  # KeyError for an unknown switch
    if name in os.environ:
        return os.environ[name]
    return file_values().get(name, default)
