"""Model shape constants, as in the reference's tinygiant/_constants.py (Qwen3-30B-A3B),
plus the DeepSeek-V3-like MoE shape of the large expert-parallel configuration."""
N_LAYERS = 48
N_HEADS = 32
N_KV_HEADS = 4
HEAD_DIM = 128
EMBED_DIM = 2048
N_EXPERTS = 128
N_EXPERTS_USED = 8
EXPERT_INTERMEDIATE = 768
VOCAB_SIZE = 151936
ROPE_BASE = 1_000_000.0
RMS_EPS = 1e-6
GQA_RATIO = N_HEADS // N_KV_HEADS
EXPERT_KEYS_ORDER = ["gate", "up", "down"]

# Q4_0 / Q8_0 block geometry (ggml)
QK = 32
Q4_0_BYTES = 18
Q8_0_BYTES = 34

# DeepSeek-V3-like MoE shape (routed experts + one shared expert)
DSV3_EMBED_DIM = 7168
DSV3_EXPERT_INTERMEDIATE = 2048
DSV3_N_EXPERTS = 256
DSV3_N_EXPERTS_USED = 8
DSV3_N_LAYERS = 58


def expert_bytes(embed: int = EMBED_DIM, inter: int = EXPERT_INTERMEDIATE) -> int:
    """Bytes of one Q4_0 expert blob gate | up | down."""
    return 3 * inter * (embed // QK) * Q4_0_BYTES
