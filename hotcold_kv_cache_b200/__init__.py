"""B200-native hot/cold KV decode path (placeholder during bring-up)."""
