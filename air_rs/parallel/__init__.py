"""air_rs.parallel."""
