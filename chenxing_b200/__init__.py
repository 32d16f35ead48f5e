"""chenxing_b200 — B200-native KV-cache hot path for Chenxing (placeholder, filled below)."""
