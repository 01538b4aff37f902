"""Weight formats: the 4-bit block format, block-scaled fp8, safetensors and GGUF readers."""
