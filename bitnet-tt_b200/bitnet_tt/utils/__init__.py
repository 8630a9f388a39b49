"""Host utilities: quantisers, RoPE tables, weight loading."""
