"""air_rs.runtime."""
