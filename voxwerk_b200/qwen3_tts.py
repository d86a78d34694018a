"""Qwen3-TTS configuration constants used on the sampling path (src/Voxwerk/Talker/Qwen3TtsConfig.cs,
TalkerGenerator.cs).  Pure Python: importing it loads no native library."""

VOCAB_SIZE = 3072          # Qwen3TtsConfig.cs:28 talker codec vocabulary
NUM_CODE_GROUPS = 16       # Qwen3TtsConfig.cs:31
CODEC_EOS_ID = 2150        # Qwen3TtsConfig.cs:34
CP_VOCAB_SIZE = 2048       # Qwen3TtsConfig.cs:49 code-predictor vocabulary
SUPPRESS_SPAN = 1024       # TalkerGenerator.cs:247: ids [V - 1024, V) except EOS
MIN_NEW_TOKENS = 2         # TalkerGenerator.cs:248: EOS suppressed while t < 2
