"""air_rs.kv."""
