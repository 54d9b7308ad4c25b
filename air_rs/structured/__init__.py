"""air_rs.structured."""
