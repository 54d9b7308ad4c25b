"""air_rs.spec."""
