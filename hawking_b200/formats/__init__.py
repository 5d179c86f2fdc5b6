"""Model containers: GGUF (ggml block quants), .gravity shards, HGRAV* mixed codecs."""
