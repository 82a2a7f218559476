"""Dataset preparation: raw benchmark files -> the JSONL rows the workflows read."""
