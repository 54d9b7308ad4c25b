"""air_rs.quant."""
